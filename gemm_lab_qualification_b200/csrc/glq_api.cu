// glq_api.cu -- the extern "C" boundary of libglq.so (declared in
// include/glq.h): argument validation, path planning, per-device set-up,
// dispatch to the kernels, path/status names and the device error word.
//
// Nothing here allocates device memory; the only device-resident state is the
// per-device sticky error word below.  No C++ exception crosses the boundary.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <mutex>

#include "glq_internal.h"

namespace glq {
namespace {

// Sticky error word raised by kernels whose bounded waits expired.
__device__ unsigned int g_device_error_word;

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int status = GLQ_OK;  // glq_status of the set-up
  int sm_count = 148;
  unsigned int* error_word = nullptr;
};

DeviceState g_devices[kMaxDevices];

int device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return GLQ_ERR_DEVICE;
  DeviceState& st = g_devices[dev];
  std::call_once(st.once, [&st, dev] {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      st.status = GLQ_ERR_DEVICE;
      return;
    }
    // The kernels are built for sm_100a only (compute capability 10.0).
    if (major != 10 || minor != 0) {
      st.status = GLQ_ERR_DEVICE;
      return;
    }
    st.sm_count = sms > 0 ? sms : 148;
    void* word = nullptr;
    if (cudaGetSymbolAddress(&word, g_device_error_word) != cudaSuccess ||
        tc_prepare_device() != cudaSuccess || gemv_prepare_device() != cudaSuccess) {
      cudaGetLastError();
      st.status = GLQ_ERR_CUDA;
      return;
    }
    st.error_word = static_cast<unsigned int*>(word);
    st.status = GLQ_OK;
  });
  *out = &st;
  return st.status;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int auto_split(int64_t tiles, int64_t k_blocks, int sm_count) {
  int64_t s = sm_count / std::max<int64_t>(tiles, 1);
  s = std::min<int64_t>(s, kMaxAutoSplit);
  s = std::min<int64_t>(s, k_blocks);
  // Each split keeps at least two K blocks so the pipeline has depth.
  while (s > 1 && k_blocks / s < 2) --s;
  return static_cast<int>(std::max<int64_t>(s, 1));
}

int validate(int dtype, int epilogue, int64_t m, int64_t n, int64_t k, int split_k) {
  if (dtype != GLQ_DTYPE_F16 && dtype != GLQ_DTYPE_BF16) return GLQ_ERR_INVALID_ARGUMENT;
  if (epilogue < GLQ_EPILOGUE_NONE || epilogue > GLQ_EPILOGUE_BIAS_SILU) return GLQ_ERR_INVALID_ARGUMENT;
  if (m < 0 || n < 0 || k < 0) return GLQ_ERR_SHAPE;
  if (m > INT_MAX || n > INT_MAX || k > INT_MAX) return GLQ_ERR_SHAPE;
  if (split_k < 0 || split_k > GLQ_MAX_SPLIT) return GLQ_ERR_SPLIT;
  return GLQ_OK;
}

// Static scratch of glq_linear_gather_static: the fused gather's arrival
// counters, one word per slot, for callers that cannot allocate.  Host code
// must not use this name as a device address; static_gather_scratch() looks
// the address up once per device.
static __device__ __align__(256) unsigned int g_static_gather_scratch[GLQ_STATIC_GATHER_SLOTS];

struct StaticScratchState {
  std::once_flag once;
  int status = GLQ_OK;
  unsigned int* ptr = nullptr;
};

StaticScratchState g_static_scratch[kMaxDevices];

// Device address of g_static_gather_scratch on the current device (looked
// up once per device, with that device current).  Nothing is written here:
// every call clears its own slot on its stream.
int static_gather_scratch(unsigned int** out) {
  DeviceState* dev_state = nullptr;
  const int v = device_state(&dev_state);
  if (v != GLQ_OK) return v;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_DEVICE;
  }
  StaticScratchState& st = g_static_scratch[dev];
  std::call_once(st.once, [&st] {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_gather_scratch) != cudaSuccess) {
      cudaGetLastError();
      st.status = GLQ_ERR_CUDA;
      return;
    }
    st.ptr = static_cast<unsigned int*>(ptr);
    st.status = GLQ_OK;
  });
  *out = st.ptr;
  return st.status;
}

}  // namespace

OperandLayout classify(const Problem& p) {
  constexpr int64_t esz = 2;
  OperandLayout L;
  // W = B^T is K-contiguous (a linear layer's weight) or N-contiguous (the
  // lab's B = [K, N] row-major); anything else is strided.
  L.a_unit = p.a_cs == 1 || p.k == 1;
  L.w_kmajor = p.b_ks == 1 || p.k == 1;
  L.w_mnmajor = !L.w_kmajor && (p.b_ns == 1 || p.n == 1);
  // TMA / 128-bit loads: 16-byte aligned bases and row pitches, rows that do
  // not overlap.
  L.a_ok = L.a_unit && aligned16(p.a) &&
           (p.m == 1 || (p.a_rs > 0 && (p.a_rs * esz) % 16 == 0 && p.a_rs >= p.k));
  L.w_ok = (L.w_kmajor || L.w_mnmajor) && aligned16(p.b) &&
           (L.w_kmajor ? (p.n == 1 || (p.b_ns > 0 && (p.b_ns * esz) % 16 == 0 && p.b_ns >= p.k))
                       : (p.b_ks > 0 && (p.b_ks * esz) % 16 == 0 && p.b_ks >= p.n));
  return L;
}

int raw_operands(const Problem& p, const OperandLayout& L) {
  if (L.w_ok && L.a_ok) return 0;
  if (!L.a_unit || !L.w_kmajor || p.require_tc || small_problem(p.m, p.n, p.k)) return -1;
  RawClasses rc;
  int raw = 0;
  if (!L.w_ok) {
    if (!raw_classes(p.b, p.n, p.k, p.b_ns, &rc)) return -1;
    raw |= kRawW;
  }
  if (!L.a_ok) {
    if (!raw_classes(p.a, p.m, p.k, p.a_rs, &rc)) return -1;
    raw |= kRawA;
  }
  return raw;
}

bool repack_plan(const Problem& p, RepackPlan* r) {
  *r = RepackPlan();
  // Small problems run the small kernel on the operands as they are, and
  // the tcgen05 kernel aligns K-contiguous rows itself up to
  // kRawCopyAboveTokens tokens.
  if (p.m <= 0 || p.n <= 0 || p.k <= 0 || small_problem(p.m, p.n, p.k)) return false;
  const OperandLayout L = classify(p);
  const int raw = raw_operands(p, L);
  if (raw == 0 || (raw > 0 && p.m <= kRawCopyAboveTokens)) return false;
  auto bytes = [](int64_t rows, int64_t cols) {
    return (static_cast<size_t>(rows) * static_cast<size_t>(repack_pitch(cols)) * 2u + 255u) / 256u * 256u;
  };
  r->a = !L.a_ok;
  r->w = !L.w_ok;
  r->w_mn = L.w_mnmajor;
  if (r->a) r->a_bytes = bytes(p.m, p.k);
  if (r->w) r->w_bytes = r->w_mn ? bytes(p.k, p.n) : bytes(p.n, p.k);
  return r->a || r->w;
}

Problem repacked_problem(const Problem& p, const RepackPlan& r, void* workspace) {
  Problem q = p;
  unsigned char* base = static_cast<unsigned char*>(workspace);
  if (r.a) {
    q.a = base;
    q.a_rs = repack_pitch(p.k);
    q.a_cs = 1;
  }
  if (r.w) {
    q.b = base + r.a_bytes;
    if (r.w_mn) {
      q.b_ks = repack_pitch(p.n);
      q.b_ns = 1;
    } else {
      q.b_ks = 1;
      q.b_ns = repack_pitch(p.k);
    }
    // The copy is written by the kernel just before: the GEMM must not read
    // W ahead of its grid-dependency wait.
    q.flags &= ~static_cast<unsigned int>(GLQ_FLAG_STATIC_WEIGHTS);
  } else if (r.a) {
    // Only A is copied.  W is not written by the copy kernel, and the copy
    // kernel waits for its own predecessor before it lets the GEMM launch, so
    // the GEMM may stream W before its dependency wait (as with static
    // weights): the weight stream overlaps the copy of A.
    q.flags |= static_cast<unsigned int>(GLQ_FLAG_STATIC_WEIGHTS);
  }
  return q;
}

cudaError_t launch_repacks(const Problem& p, const RepackPlan& r, void* workspace, int sm_count, cudaStream_t s) {
  unsigned char* base = static_cast<unsigned char*>(workspace);
  cudaError_t e = cudaSuccess;
  if (r.a) e = launch_repack(p.a, p.m, p.k, p.a_rs, p.a_cs, base, sm_count, s);
  if (e == cudaSuccess && r.w) {
    // K-contiguous copy [N, K] unless B is N-contiguous ([K, N] copy).
    e = r.w_mn ? launch_repack(p.b, p.k, p.n, p.b_ks, p.b_ns, base + r.a_bytes, sm_count, s)
               : launch_repack(p.b, p.n, p.k, p.b_ns, p.b_ks, base + r.a_bytes, sm_count, s);
  }
  return e;
}

int plan_problem(const Problem& p, int split_k, int sm_count, Choice* c) {
  c->split = 1;
  c->tile_t = 0;
  c->tile_n = 128;
  c->stages = 0;
  c->kps = 1;
  c->w_mn = 0;
  c->raw = 0;
  if (p.m == 0 || p.n == 0) {
    c->path = GLQ_PATH_EMPTY;
    c->kernel = kKernelNone;
    return GLQ_OK;
  }
  if (p.k == 0) {
    c->path = GLQ_PATH_ZERO_K;
    c->kernel = kKernelFill;
    return GLQ_OK;
  }
  const OperandLayout L = classify(p);
  if (!L.a_unit || (!L.w_kmajor && !L.w_mnmajor)) {
    c->path = GLQ_PATH_STRIDED;
    c->kernel = small_problem(p.m, p.n, p.k) ? kKernelSmall : kKernelGeneric;
    return GLQ_OK;
  }
  // K-contiguous rows that TMA cannot address (odd K, a row pitch or base
  // off 16 bytes) in either operand: the tcgen05 kernel loads them by row
  // class and aligns them in shared memory (no copy, no workspace).
  const int raw = raw_operands(p, L);
  const bool staged = raw > 0;
  if (raw < 0) {
    c->path = GLQ_PATH_UNALIGNED;
    c->kernel = small_problem(p.m, p.n, p.k) ? kKernelSmall : kKernelGeneric;
    return GLQ_OK;
  }
  c->w_mn = L.w_mnmajor ? 1 : 0;
  c->raw = staged ? raw : 0;
  // M = 1 runs a GEMV, except for a forced split of 4 or more: the register
  // GEMV then holds one or two rows per block and every block re-stages all
  // of A (19 us at S = 8 vs 9.9 us for the tcgen05 split, which writes the
  // same [S, 1, N] FP32 partials).
  if (p.m == 1 && L.w_kmajor && !p.require_tc && split_k < 4 && !staged) {
    const int sms = sm_count > 0 ? sm_count : 148;
    // The ring GEMV holds a whole SM per CTA, so with static weights (where a
    // call's weight stream should start while its predecessor drains) the
    // register GEMV, whose blocks can be resident early, is faster.
    const bool ring = split_k <= 1 && (p.flags & GLQ_FLAG_STATIC_WEIGHTS) == 0 && gemv_ring_fits(p.n, p.k, sms);
    c->kernel = ring ? kKernelGemvRing : kKernelGemv;
    c->split = split_k > 0 ? split_k : 1;
    c->path = (p.k % 8 != 0) ? GLQ_PATH_TAIL : GLQ_PATH_GEMV_M1;
    return GLQ_OK;
  }
  c->kernel = kKernelTc;
  c->tile_t = tc_token_tile(p.m);
  c->tile_n = staged ? 128 : tc_tile_rows(p.m, p.n);  // raw-staged operands use 128-row tiles
  const int64_t k_blocks = tc_k_blocks(p.k);
  const int64_t tiles = ((p.n + c->tile_n - 1) / c->tile_n) * ((p.m + c->tile_t - 1) / c->tile_t);
  const int sms = sm_count > 0 ? sm_count : 148;
  int s = split_k > 0 ? split_k : auto_split(tiles, k_blocks, sms);
  // Two CTAs per SM with an 8-way split when that still fits one wave.
  if (split_k == 0 && c->tile_n == 128 && c->tile_t <= 32 && tiles * kPairSplit <= 2 * sms &&
      tiles * kPairSplit > static_cast<int64_t>(s) * tiles && k_blocks >= 2 * kPairSplit) {
    s = kPairSplit;
    c->stages = kPairStages;
  }
  if (split_k == kPairSplit && c->tile_n == 128 && c->tile_t <= 32) c->stages = kPairStages;
  s = static_cast<int>(std::min<int64_t>(s, k_blocks));
  c->split = std::max(s, 1);
  // Split-K tiles hold at most 128 tokens (the merge buffers must fit in the
  // drained pipeline memory).
  if (c->split > 1 && c->tile_t > 128) c->tile_t = 128;
  // Split-K tiles of 128 W rows move two K blocks per TMA operation (32 KB
  // of W) when K is whole blocks (and, for the lab's B = [K, N], N whole
  // blocks of 64 columns) and every split gets an even number of them: the
  // two-CTAs-per-SM split, and 64- or 128-token tiles.
  const bool pair = c->stages == kPairStages;
  if (c->split > 1 && c->tile_n == 128 && (!L.w_mnmajor || p.n % 64 == 0) && !staged && kPairKps == 2 && p.k % 64 == 0 &&
      k_blocks % c->split == 0 && (k_blocks / c->split) % 2 == 0 && kps2_stages(c->tile_t, pair) > 0) {
    c->kps = 2;
    c->stages = kps2_stages(c->tile_t, pair);
  }
  // Prefill-sized problems (256-token tiles, no split) with at least one
  // wave of 256 x 256 output tiles: two M = 128 MMAs per K step share the
  // token tile, doubling the FLOPs per staged byte.
  if (c->split == 1 && c->tile_t == 256 && !staged &&
      ((p.n + 255) / 256) * ((p.m + 255) / 256) >= static_cast<int64_t>(sms)) {
    c->tile_n = 256;
  }
  if (staged) {
    c->path = GLQ_PATH_TC_LDG;
  } else if (p.n % 128 != 0 || p.k % 64 != 0) {
    c->path = GLQ_PATH_TAIL;
  } else if (c->w_mn) {
    c->path = GLQ_PATH_TC_KN;
  } else {
    c->path = c->split > 1 ? GLQ_PATH_TC_SPLITK : GLQ_PATH_TC;
  }
  return GLQ_OK;
}

// A validated, planned fused-gather call (glq_linear_gather and its
// allocation-free variant share it): nothing runs on the device until
// launch_gather.
struct GatherCall {
  Problem p;
  Gather g;
  Choice c;
  DeviceState* dev;
};

int prepare_gather(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride, const void* B,
                   int64_t b_k_stride, int64_t b_n_stride, const void* bias, int epilogue, void* const* y_ranks,
                   int64_t y_row_stride, int64_t y_col_offset, int64_t M, int64_t N, int64_t K, int split_k, int rank,
                   int world, uint64_t* const* signal_ranks, uint64_t epoch, unsigned int flags, bool no_counter,
                   GatherCall* call) {
  int v = validate(dtype, epilogue, M, N, K, split_k);
  if (v != GLQ_OK) return v;
  if ((flags & ~(GLQ_FLAG_NO_PDL | GLQ_FLAG_STATIC_WEIGHTS)) != 0) return GLQ_ERR_INVALID_ARGUMENT;
  if (world < 1 || world > GLQ_MAX_RANKS || rank < 0 || rank >= world) return GLQ_ERR_INVALID_ARGUMENT;
  if (M <= 0 || N <= 0 || K <= 0) return GLQ_ERR_SHAPE;
  if (A == nullptr || B == nullptr || y_ranks == nullptr || signal_ranks == nullptr || no_counter || epoch == 0) {
    return GLQ_ERR_INVALID_ARGUMENT;
  }
  if (epilogue != GLQ_EPILOGUE_NONE && bias == nullptr) return GLQ_ERR_INVALID_ARGUMENT;
  if (y_col_offset < 0 || y_row_stride < y_col_offset + N) return GLQ_ERR_OUTPUT_LAYOUT;
  // 16-bit elements: every element pointer is 2-byte aligned (the kernels'
  // 16-bit loads and stores fault on an odd address).
  auto odd = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 1u) != 0; };
  if (odd(A) || odd(B) || (bias != nullptr && odd(bias))) return GLQ_ERR_INVALID_ARGUMENT;
  constexpr int64_t esz = 2;
  Gather& g = call->g;
  g = Gather{};
  g.rank = rank;
  g.world = world;
  for (int r = 0; r < world; ++r) {
    if (y_ranks[r] == nullptr || signal_ranks[r] == nullptr || odd(y_ranks[r])) return GLQ_ERR_INVALID_ARGUMENT;
    g.y[r] = static_cast<char*>(y_ranks[r]) + y_col_offset * esz;
    g.signal[r] = reinterpret_cast<unsigned long long*>(signal_ranks[r]);
  }
  g.counter = nullptr;
  g.epoch = static_cast<unsigned long long>(epoch);

  Problem& p = call->p;
  p = Problem{};
  p.dtype = dtype;
  p.a = A;
  p.a_rs = a_row_stride;
  p.a_cs = a_col_stride;
  p.b = B;
  p.b_ks = b_k_stride;
  p.b_ns = b_n_stride;
  p.bias = bias;
  p.epilogue = epilogue;
  p.y = g.y[rank];
  p.ldy = y_row_stride;
  p.m = M;
  p.n = N;
  p.k = K;
  p.partial = nullptr;
  p.flags = flags;
  p.require_tc = 1;

  v = device_state(&call->dev);
  if (v != GLQ_OK) return v;
  v = plan_problem(p, split_k, call->dev->sm_count, &call->c);
  if (v != GLQ_OK) return v;
  if (call->c.kernel != kKernelTc) return GLQ_ERR_INVALID_ARGUMENT;
  return GLQ_OK;
}

int launch_gather(GatherCall* call, unsigned int* counter, cudaStream_t s, int* path_out, int* split_out) {
  call->g.counter = counter;
  const Choice& c = call->c;
  const cudaError_t e =
      launch_tc(call->p, c.split, c.tile_t, c.tile_n, c.stages, c.kps, c.w_mn, &call->g, call->dev->error_word, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_CUDA;
  }
  if (path_out) *path_out = c.path;
  if (split_out) *split_out = c.split;
  return GLQ_OK;
}

}  // namespace glq

using glq::Choice;
using glq::Problem;

extern "C" {

int glq_plan(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride, const void* B,
             int64_t b_k_stride, int64_t b_n_stride, int64_t y_row_stride, int64_t M, int64_t N,
             int64_t K, int split_k, int sm_count, int* path_out, int* split_out) {
  const int v = glq::validate(dtype, GLQ_EPILOGUE_NONE, M, N, K, split_k);
  if (v != GLQ_OK) return v;
  if (M > 1 && N > 0 && y_row_stride < N) return GLQ_ERR_OUTPUT_LAYOUT;
  Problem p = {};
  p.dtype = dtype;
  p.a = A;
  p.a_rs = a_row_stride;
  p.a_cs = a_col_stride;
  p.b = B;
  p.b_ks = b_k_stride;
  p.b_ns = b_n_stride;
  p.ldy = y_row_stride;
  p.m = M;
  p.n = N;
  p.k = K;
  Choice c;
  const int r = glq::plan_problem(p, split_k, sm_count, &c);
  if (r != GLQ_OK) return r;
  if (path_out) *path_out = c.path;
  if (split_out) *split_out = c.split;
  return GLQ_OK;
}

int glq_linear(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride, const void* B,
               int64_t b_k_stride, int64_t b_n_stride, const void* bias, int epilogue, void* Y,
               int64_t y_row_stride, int64_t M, int64_t N, int64_t K, int split_k, void* workspace,
               size_t workspace_bytes, void* stream, int* path_out, int* split_out) {
  return glq_linear_ex(dtype, A, a_row_stride, a_col_stride, B, b_k_stride, b_n_stride, bias, epilogue, Y,
                       y_row_stride, M, N, K, split_k, workspace, workspace_bytes, stream, 0u, path_out,
                       split_out);
}

int glq_linear_ex(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride, const void* B,
                  int64_t b_k_stride, int64_t b_n_stride, const void* bias, int epilogue, void* Y,
                  int64_t y_row_stride, int64_t M, int64_t N, int64_t K, int split_k, void* workspace,
                  size_t workspace_bytes, void* stream, unsigned int flags, int* path_out, int* split_out) {
  int v = glq::validate(dtype, epilogue, M, N, K, split_k);
  if (v != GLQ_OK) return v;
  if ((flags & ~(GLQ_FLAG_NO_PDL | GLQ_FLAG_STATIC_WEIGHTS)) != 0) return GLQ_ERR_INVALID_ARGUMENT;
  if (M > 0 && N > 0) {
    if (Y == nullptr) return GLQ_ERR_INVALID_ARGUMENT;
    if (M > 1 && y_row_stride < N) return GLQ_ERR_OUTPUT_LAYOUT;
    if (epilogue != GLQ_EPILOGUE_NONE && bias == nullptr) return GLQ_ERR_INVALID_ARGUMENT;
    if (K > 0 && (A == nullptr || B == nullptr)) return GLQ_ERR_INVALID_ARGUMENT;
    // 16-bit elements: every element pointer is 2-byte aligned.
    auto odd = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 1u) != 0; };
    if (odd(Y) || (bias != nullptr && odd(bias)) || (K > 0 && (odd(A) || odd(B)))) return GLQ_ERR_INVALID_ARGUMENT;
  }
  Problem p = {};
  p.dtype = dtype;
  p.a = A;
  p.a_rs = a_row_stride;
  p.a_cs = a_col_stride;
  p.b = B;
  p.b_ks = b_k_stride;
  p.b_ns = b_n_stride;
  p.bias = bias;
  p.epilogue = epilogue;
  p.y = Y;
  p.ldy = y_row_stride;
  p.m = M;
  p.n = N;
  p.k = K;
  p.partial = nullptr;
  p.flags = flags;

  Choice c;
  if (path_out) *path_out = GLQ_PATH_EMPTY;
  if (split_out) *split_out = 1;
  if (M == 0 || N == 0) {
    return glq::plan_problem(p, split_k, 0, &c);
  }
  glq::DeviceState* dev = nullptr;
  v = glq::device_state(&dev);
  if (v != GLQ_OK) return v;
  v = glq::plan_problem(p, split_k, dev->sm_count, &c);
  if (v != GLQ_OK) return v;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Strided operands, unaligned ones the tcgen05 kernel cannot stage itself
  // (such as the lab's B = [K, N] with rows off 16 bytes), and unaligned
  // K-contiguous ones of problems above kRawCopyAboveTokens tokens, with a
  // workspace that holds their aligned copies: repack, then plan the copies
  // (tcgen05 / GEMV instead of the generic or raw-staged kernel).
  glq::RepackPlan rp;
  const bool copies = c.kernel == glq::kKernelGeneric || (c.raw != 0 && p.m > glq::kRawCopyAboveTokens);
  const bool repack = copies && workspace != nullptr &&
                      glq::aligned16(workspace) && glq::repack_plan(p, &rp) && workspace_bytes >= rp.bytes();
  if (repack) {
    if (glq::launch_repacks(p, rp, workspace, dev->sm_count, s) != cudaSuccess) {
      cudaGetLastError();
      return GLQ_ERR_CUDA;
    }
    p = glq::repacked_problem(p, rp, workspace);
    v = glq::plan_problem(p, split_k, dev->sm_count, &c);
    if (v != GLQ_OK) return v;
  } else if (workspace != nullptr && c.split > 1) {
    // The FP32 partials are stored as floats: a 4-byte aligned buffer.
    const size_t need = static_cast<size_t>(c.split) * static_cast<size_t>(M) * static_cast<size_t>(N) * sizeof(float);
    if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) return GLQ_ERR_WORKSPACE;
    p.partial = static_cast<float*>(workspace);
  }
  p.raw = c.raw;
  cudaError_t e = cudaSuccess;
  switch (c.kernel) {
    case glq::kKernelFill: e = glq::launch_fill(p, s); break;
    case glq::kKernelGemv: e = glq::launch_gemv(p, c.split, dev->error_word, s); break;
    case glq::kKernelGemvRing: e = glq::launch_gemv_ring(p, dev->error_word, s, dev->sm_count); break;
    case glq::kKernelTc:
      e = glq::launch_tc(p, c.split, c.tile_t, c.tile_n, c.stages, c.kps, c.w_mn, nullptr, dev->error_word, s);
      break;
    case glq::kKernelGeneric: e = glq::launch_generic(p, s); break;
    case glq::kKernelSmall: e = glq::launch_small(p, s); break;
    default: break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_CUDA;
  }
  if (path_out) *path_out = repack ? GLQ_PATH_REPACKED : c.path;
  if (split_out) *split_out = (c.kernel == glq::kKernelGeneric || c.kernel == glq::kKernelSmall) ? 1 : c.split;
  return GLQ_OK;
}

size_t glq_linear_workspace_bytes(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride,
                                  const void* B, int64_t b_k_stride, int64_t b_n_stride, int64_t M, int64_t N,
                                  int64_t K) {
  if (glq::validate(dtype, GLQ_EPILOGUE_NONE, M, N, K, 0) != GLQ_OK) return 0;
  Problem p = {};
  p.dtype = dtype;
  p.a = A;
  p.a_rs = a_row_stride;
  p.a_cs = a_col_stride;
  p.b = B;
  p.b_ks = b_k_stride;
  p.b_ns = b_n_stride;
  p.m = M;
  p.n = N;
  p.k = K;
  glq::RepackPlan rp;
  return glq::repack_plan(p, &rp) ? rp.bytes() : 0;
}

int glq_linear_gather(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride, const void* B,
                      int64_t b_k_stride, int64_t b_n_stride, const void* bias, int epilogue, void* const* y_ranks,
                      int64_t y_row_stride, int64_t y_col_offset, int64_t M, int64_t N, int64_t K, int split_k,
                      int rank, int world, uint64_t* const* signal_ranks, unsigned int* counter, uint64_t epoch,
                      void* stream, unsigned int flags, int* path_out, int* split_out) {
  if (path_out) *path_out = GLQ_PATH_EMPTY;
  if (split_out) *split_out = 1;
  glq::GatherCall call;
  const int v = glq::prepare_gather(dtype, A, a_row_stride, a_col_stride, B, b_k_stride, b_n_stride, bias, epilogue,
                                    y_ranks, y_row_stride, y_col_offset, M, N, K, split_k, rank, world,
                                    signal_ranks, epoch, flags, counter == nullptr, &call);
  if (v != GLQ_OK) return v;
  return glq::launch_gather(&call, counter, static_cast<cudaStream_t>(stream), path_out, split_out);
}

int glq_linear_gather_static(int dtype, const void* A, int64_t a_row_stride, int64_t a_col_stride,
                             const void* B, int64_t b_k_stride, int64_t b_n_stride, const void* bias,
                             int epilogue, void* const* y_ranks, int64_t y_row_stride, int64_t y_col_offset,
                             int64_t M, int64_t N, int64_t K, int split_k, int rank, int world,
                             uint64_t* const* signal_ranks, int counter_slot, uint64_t epoch, void* stream,
                             unsigned int flags, int* path_out, int* split_out) {
  if (path_out) *path_out = GLQ_PATH_EMPTY;
  if (split_out) *split_out = 1;
  if (counter_slot < 0 || counter_slot >= GLQ_STATIC_GATHER_SLOTS) return GLQ_ERR_SCRATCH;
  // Everything that can refuse the call runs before the slot is touched, so a
  // rejected call leaves a slot that another stream may be using alone.
  glq::GatherCall call;
  int v = glq::prepare_gather(dtype, A, a_row_stride, a_col_stride, B, b_k_stride, b_n_stride, bias, epilogue,
                              y_ranks, y_row_stride, y_col_offset, M, N, K, split_k, rank, world, signal_ranks,
                              epoch, flags, false, &call);
  if (v != GLQ_OK) return v;
  unsigned int* scratch = nullptr;
  v = glq::static_gather_scratch(&scratch);
  if (v != GLQ_OK) return v;
  unsigned int* counter = scratch + counter_slot;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The kernel leaves the counter at zero, but a call whose wait expired may
  // not have: start every call from zero, in stream order.
  if (cudaMemsetAsync(counter, 0, sizeof(unsigned int), s) != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_CUDA;
  }
  return glq::launch_gather(&call, counter, s, path_out, split_out);
}

int glq_linear_f16(const void* A, int64_t lda, int64_t a_col_stride, const void* B,
                   int64_t b_row_stride, int64_t b_col_stride, const void* bias, void* Y, int64_t ldy,
                   int M, int N, int K, int split_k, void* workspace, size_t workspace_bytes,
                   void* stream, int* path_out) {
  return glq_linear(GLQ_DTYPE_F16, A, lda, a_col_stride, B, b_row_stride, b_col_stride, bias,
                    bias != nullptr ? GLQ_EPILOGUE_BIAS_SILU : GLQ_EPILOGUE_NONE, Y, ldy, M, N, K,
                    split_k, workspace, workspace_bytes, stream, path_out, nullptr);
}

int glq_matmul(int dtype, const void* a, const void* b, void* c, int m, int n, int k, void* stream) {
  return glq_linear(dtype, a, k, 1, b, n, 1, nullptr, GLQ_EPILOGUE_NONE, c, n, m, n, k, 0, nullptr, 0,
                    stream, nullptr, nullptr);
}

int glq_splitk_matmul(int dtype, const void* a, const void* b, void* c, int m, int n, int k,
                      float* partial, int splits, void* stream) {
  if (splits < 1 || splits > GLQ_MAX_SPLIT) return GLQ_ERR_SPLIT;
  const size_t bytes = partial != nullptr ? glq_workspace_bytes(m, n, k, splits) : 0;
  return glq_linear(dtype, a, k, 1, b, n, 1, nullptr, GLQ_EPILOGUE_NONE, c, n, m, n, k, splits, partial,
                    bytes, stream, nullptr, nullptr);
}

size_t glq_workspace_bytes(int64_t M, int64_t N, int64_t K, int split_k) {
  if (M <= 0 || N <= 0 || K <= 0 || split_k < 0 || split_k > GLQ_MAX_SPLIT) return 0;
  // The larger of the plans of a K-contiguous W (row pitch K) and an
  // N-contiguous B = [K, N] (row pitch N); they differ only at M == 1.
  Problem p = {};
  p.dtype = GLQ_DTYPE_F16;
  p.a_rs = K;
  p.a_cs = 1;
  p.b_ks = 1;
  p.b_ns = K;
  p.ldy = N;
  p.m = M;
  p.n = N;
  p.k = K;
  int split = 1;
  for (int layout = 0; layout < 2; ++layout) {
    if (layout == 1) {
      p.b_ks = N;
      p.b_ns = 1;
    }
    Choice c;
    if (glq::plan_problem(p, split_k, 0, &c) == GLQ_OK) split = std::max(split, c.split);
  }
  if (split <= 1) return 0;
  return static_cast<size_t>(split) * static_cast<size_t>(M) * static_cast<size_t>(N) * sizeof(float);
}

const char* glq_path_name(int path) {
  switch (path) {
    case GLQ_PATH_EMPTY: return "empty";
    case GLQ_PATH_ZERO_K: return "zero_k";
    case GLQ_PATH_GEMV_M1: return "gemv_m1";
    case GLQ_PATH_TC: return "tc_tcgen05";
    case GLQ_PATH_TC_SPLITK: return "tc_splitk";
    case GLQ_PATH_TAIL: return "tail";
    case GLQ_PATH_STRIDED: return "strided";
    case GLQ_PATH_UNALIGNED: return "unaligned";
    case GLQ_PATH_TC_KN: return "tc_kn";
    case GLQ_PATH_REPACKED: return "repacked";
    case GLQ_PATH_TC_LDG: return "tc_ldg";
    default: return "unknown";
  }
}

const char* glq_status_string(int status) {
  switch (status) {
    case GLQ_OK: return "ok";
    case GLQ_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, dtype or epilogue)";
    case GLQ_ERR_SHAPE: return "invalid shape or stride";
    case GLQ_ERR_SPLIT: return "split_k must be in 0..8";
    case GLQ_ERR_WORKSPACE: return "workspace smaller than split * M * N * 4 bytes, or not 4-byte aligned";
    case GLQ_ERR_OUTPUT_LAYOUT: return "output row stride smaller than N";
    case GLQ_ERR_CUDA: return "CUDA runtime or driver call failed";
    case GLQ_ERR_DEVICE: return "no usable device: the kernels need a compute capability 10.0 (sm_100a) GPU";
    case GLQ_ERR_DEVICE_TIMEOUT: return "an in-kernel bounded wait expired";
    case GLQ_ERR_SCRATCH: return "counter_slot outside the library's static scratch (0..GLQ_STATIC_GATHER_SLOTS-1)";
    default: return "unknown status";
  }
}

int glq_device_error(unsigned int* word_out, int clear) {
  if (word_out == nullptr) return GLQ_ERR_INVALID_ARGUMENT;
  glq::DeviceState* dev = nullptr;
  const int v = glq::device_state(&dev);
  if (v != GLQ_OK) return v;
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_CUDA;
  }
  unsigned int word = 0;
  if (cudaMemcpy(&word, dev->error_word, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return GLQ_ERR_CUDA;
  }
  if (clear && word != 0) {
    if (cudaMemset(dev->error_word, 0, sizeof(word)) != cudaSuccess) {
      cudaGetLastError();
      return GLQ_ERR_CUDA;
    }
  }
  *word_out = word;
  return GLQ_OK;
}

int glq_abi_version(void) { return GLQ_ABI_VERSION; }

const char* glq_build_target(void) { return "sm_100a"; }

}  // extern "C"
