// glq_gemv.cu -- M = 1 linear kernel: y[n] = epilogue(sum_k a[k] * W[n, k]).
//
// One token costs 2 flops per weight element, far below the tensor-core
// ridge, so the weight stream is the whole cost.  Each warp reduces one W row
// (or one of `split` contiguous K ranges of it): lanes issue 128-bit
// streaming loads (ld.global.nc.L1::no_allocate) of consecutive 16-byte
// chunks, UNROLL chunks per lane in flight before any arithmetic (registers
// capped so four 256-thread blocks fit per SM: N = 4096 rows is one wave on
// 148 SMs), accumulate
// in FP32, and reduce with a fixed xor-shuffle tree.  With split > 1 the
// partial sums of one row are merged by its first warp in split order
// 0..split-1 through shared memory, so the result is deterministic; the
// optional FP32 partials are written in the lab's [split, 1, N] layout.
//
// Launched with programmatic dependent launch (see glq.h, glq_flags).
//
// Reference counterpart: the M = 1 rows of the split-K and tiled kernels
// (csrc/ptx_mma.cuh:502-770, kernels.py:324-393); the CTest case
// 1x4096x4096 (CMakeLists.txt:45-51) exercises this shape.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "glq_internal.h"
#include "glq_ptx.cuh"

namespace glq {
namespace {

struct GemvArgs {
  const void* a;
  const void* w;
  long long ldw;
  const void* bias;
  int epilogue;
  void* y;
  int n;
  int k;
  int split;
  int rows_per_block;
  float* partial;
  unsigned int flags;
  int a_in_smem;  // 1: the block stages A (K/8 16-byte chunks) in dynamic shared memory
};

__device__ __forceinline__ float apply_epilogue(float acc, float bias, int epilogue) {
  if (epilogue == GLQ_EPILOGUE_NONE) return acc;
  const float v = acc + bias;
  if (epilogue == GLQ_EPILOGUE_BIAS) return v;
  return __fdividef(v, 1.0f + __expf(-v));
}

template <typename T>
struct Vec;

template <>
struct Vec<__half> {
  __device__ static float2 pair(uint32_t bits) {
    __half2 h = *reinterpret_cast<const __half2*>(&bits);
    return __half22float2(h);
  }
  __device__ static float to_f(__half v) { return __half2float(v); }
  __device__ static __half from_f(float v) { return __float2half_rn(v); }
};

template <>
struct Vec<__nv_bfloat16> {
  __device__ static float2 pair(uint32_t bits) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&bits);
    return __bfloat1622float2(h);
  }
  __device__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T>
__device__ __forceinline__ void dot8(const uint4& w, const uint4& a, float& acc0, float& acc1) {
  const float2 w0 = Vec<T>::pair(w.x), a0 = Vec<T>::pair(a.x);
  const float2 w1 = Vec<T>::pair(w.y), a1 = Vec<T>::pair(a.y);
  const float2 w2 = Vec<T>::pair(w.z), a2 = Vec<T>::pair(a.z);
  const float2 w3 = Vec<T>::pair(w.w), a3 = Vec<T>::pair(a.w);
  acc0 = fmaf(w0.x, a0.x, acc0);
  acc1 = fmaf(w0.y, a0.y, acc1);
  acc0 = fmaf(w1.x, a1.x, acc0);
  acc1 = fmaf(w1.y, a1.y, acc1);
  acc0 = fmaf(w2.x, a2.x, acc0);
  acc1 = fmaf(w2.y, a2.y, acc1);
  acc0 = fmaf(w3.x, a3.x, acc0);
  acc1 = fmaf(w3.y, a3.y, acc1);
}

constexpr int kBlockThreadsMax = 256;
// A is staged in shared memory up to this many bytes (K <= 24576); four
// blocks per SM still fit.
constexpr size_t kGemvSmemA = 48 * 1024;

template <typename T, int UNROLL>
__global__ void __launch_bounds__(kBlockThreadsMax, 4) gemv_kernel(const GemvArgs g) {
  __shared__ float warp_sums[kBlockThreadsMax / 32];
  extern __shared__ uint4 a_smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = g.split;
  const int row_slot = warp / split;
  const int part = warp % split;
  const long long n = static_cast<long long>(blockIdx.x) * g.rows_per_block + row_slot;

  float acc0 = 0.0f, acc1 = 0.0f;
  const bool row_ok = n < g.n;
  const T* wrow = static_cast<const T*>(g.w) + (row_ok ? n : 0) * g.ldw;
  const uint4* wv = reinterpret_cast<const uint4*>(wrow);
  const uint4* av = reinterpret_cast<const uint4*>(g.a);
  const int chunks = g.k >> 3;
  const int c_begin = static_cast<int>((static_cast<long long>(part) * chunks) / split);
  const int c_end = row_ok ? static_cast<int>((static_cast<long long>(part + 1) * chunks) / split) : c_begin;
  uint4 w[UNROLL];
  auto load_w = [&](int c0) {
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int cc = c0 + u * 32;
      w[u] = cc < c_end ? ptx::ldg_stream_v4(wv + cc) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // Programmatic dependent launch: a, bias and y wait for the predecessor
  // grid; the first weight chunks may be requested before that when the
  // caller declared the weights static.
  const bool static_w = (g.flags & GLQ_FLAG_STATIC_WEIGHTS) != 0;
  if (static_w) load_w(c_begin + lane);
  ptx::grid_dependency_wait();
  ptx::grid_launch_dependents();
  // A (a few KB, resident in L2) is requested first so that its loads do not
  // queue behind the weight stream, then the first weight chunks; A is staged
  // once per block in shared memory (every warp reads all of it), then the
  // bias of this warp's row is requested, so none of these latencies lands at
  // the end.
  constexpr int kAPerThread = 2;
  uint4 a_regs[kAPerThread];
  int a_next = threadIdx.x;
  if (g.a_in_smem) {
#pragma unroll
    for (int i = 0; i < kAPerThread; ++i) {
      const int c = a_next + i * static_cast<int>(blockDim.x);
      if (c < chunks) a_regs[i] = __ldg(av + c);
    }
  }
  if (!static_w) load_w(c_begin + lane);
  if (g.a_in_smem) {
#pragma unroll
    for (int i = 0; i < kAPerThread; ++i) {
      const int c = a_next + i * static_cast<int>(blockDim.x);
      if (c < chunks) a_smem[c] = a_regs[i];
    }
    for (int c = a_next + kAPerThread * static_cast<int>(blockDim.x); c < chunks; c += blockDim.x) a_smem[c] = __ldg(av + c);
  }
  float bias_v = 0.0f;
  if (g.epilogue != GLQ_EPILOGUE_NONE && row_ok && part == 0 && lane == 0) {
    bias_v = Vec<T>::to_f(static_cast<const T*>(g.bias)[n]);
  }
  if (g.a_in_smem) __syncthreads();
  if (row_ok) {
    for (int c = c_begin + lane; c < c_end; c += 32 * UNROLL) {
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int cc = c + u * 32;
        if (cc < c_end) {
          const uint4 a = g.a_in_smem ? a_smem[cc] : __ldg(av + cc);
          dot8<T>(w[u], a, acc0, acc1);
        }
      }
      if (c + 32 * UNROLL < c_end) load_w(c + 32 * UNROLL);
    }
    if (part == split - 1 && lane == 0) {
      // K % 8 remainder, scalar, in ascending k.
      const T* a = static_cast<const T*>(g.a);
      for (int kk = chunks << 3; kk < g.k; ++kk) {
        acc0 = fmaf(Vec<T>::to_f(wrow[kk]), Vec<T>::to_f(a[kk]), acc0);
      }
    }
  }
  float acc = acc0 + acc1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) warp_sums[warp] = acc;
  __syncthreads();
  if (part == 0 && lane == 0 && n < g.n) {
    float sum = 0.0f;
    for (int p = 0; p < split; ++p) {
      const float v = warp_sums[row_slot * split + p];
      sum += v;
      if (g.partial != nullptr) g.partial[static_cast<long long>(p) * g.n + n] = v;
    }
    static_cast<T*>(g.y)[n] = Vec<T>::from_f(apply_epilogue(sum, bias_v, g.epilogue));
  }
}

// ---------------------------------------------------------------- ring GEMV
//
// M = 1 without a forced split, K % 8 == 0: the weight stream goes through
// the TMA engine instead of registers.  One CTA per SM owns a contiguous
// block of W rows; a producer lane issues 1-D bulk copies of row pieces (up
// to 8 KB) into a ring of 8 KB stages that fills most of shared memory, so
// ~190 KB per SM (all of a 32 MB weight across the GPU) is requested as soon
// as the dependency wait returns, where the register GEMV above can keep
// only two batches of 4 KB per warp in flight.  Eight consumer warps take the
// stages round-robin, each reducing one piece against A (staged once per CTA
// by the same engine) with FP32 FMAs and a fixed xor-shuffle tree; a final
// pass sums the pieces of each row in order and applies the epilogue, so the
// result is deterministic.  Every wait is bounded.
struct RingArgs {
  const void* a;
  const void* w;
  long long ldw;
  const void* bias;
  int epilogue;
  void* y;
  int n, k;
  int rows_per_cta;
  int pieces;          // pieces per row
  int piece_elems;     // elements per full piece
  int stages;
  uint32_t stage_bytes;
  uint32_t a_offset;   // shared-memory byte offsets
  uint32_t part_offset;
  uint32_t bar_offset;
  unsigned int* err;
  unsigned int flags;
};

constexpr int kRingConsumers = 8;
constexpr int kRingThreads = (kRingConsumers + 1) * 32;  // + one producer warp
constexpr int kRingPieceElems = 4096;                    // 8 KB of FP16/BF16
constexpr int kRingMaxStages = 48;
constexpr uint32_t kRingSmem = 232448;                   // 227 KB opt-in

template <typename T>
__global__ void __launch_bounds__(kRingThreads, 1) gemv_ring_kernel(const RingArgs g) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = ptx::smem_addr(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * g.rows_per_cta;
  const int rows = min(g.rows_per_cta, g.n - row0);
  const int units = rows * g.pieces;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + g.bar_offset);
  auto full = [&](int s) { return ptx::smem_addr(&bars[s]); };
  auto empty = [&](int s) { return ptx::smem_addr(&bars[g.stages + s]); };
  const uint32_t a_bar = ptx::smem_addr(&bars[2 * g.stages]);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(&bars[2 * g.stages + 1]);
  int* issued_slot = reinterpret_cast<int*>(&bars[2 * g.stages + 2]);
  float* part = reinterpret_cast<float*>(smem + g.part_offset);
  auto raise = [&](unsigned int bit) {
    atomicOr(g.err, bit);
    *abort_flag = 1;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      ptx::mbar_init(full(s), 1);
      ptx::mbar_init(empty(s), 1);
    }
    ptx::mbar_init(a_bar, 1);
    *abort_flag = 0;
    *issued_slot = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (warp == kRingConsumers) {
    // ---- producer (one lane)
    if (lane == 0) {
      const T* w = static_cast<const T*>(g.w);
      const uint64_t pol_w = ptx::policy_evict_first();
      auto issue = [&](int u) {
        const int s = u % g.stages;
        const int r = u / g.pieces;
        const int e0 = (u - r * g.pieces) * g.piece_elems;
        const uint32_t bytes = static_cast<uint32_t>(min(g.piece_elems, g.k - e0)) * 2u;
        ptx::mbar_arrive_expect_tx(full(s), bytes);
        ptx::bulk_load_1d(sbase + static_cast<uint32_t>(s) * g.stage_bytes,
                          w + static_cast<long long>(row0 + r) * g.ldw + e0, bytes, full(s), pol_w);
      };
      const int first = min(units, g.stages);
      const bool static_w = (g.flags & GLQ_FLAG_STATIC_WEIGHTS) != 0;
      if (static_w) {
        for (int u = 0; u < first; ++u) issue(u);
      }
      ptx::grid_dependency_wait();
      ptx::grid_launch_dependents();
      const uint32_t a_bytes = static_cast<uint32_t>(g.k) * 2u;
      ptx::mbar_arrive_expect_tx(a_bar, a_bytes);
      ptx::bulk_load_1d(sbase + g.a_offset, g.a, a_bytes, a_bar, ptx::policy_evict_last());
      int issued = first;
      if (!static_w) {
        for (int u = 0; u < first; ++u) issue(u);
      }
      for (int u = first; u < units; ++u) {
        const int s = u % g.stages;
        if (!ptx::mbar_wait_bounded(empty(s), static_cast<uint32_t>(u / g.stages - 1) & 1u, abort_flag,
                                    kWaitBudgetNs)) {
          raise(kErrTimeoutProducer);
          break;
        }
        issue(u);
        issued = u + 1;
      }
      *issued_slot = issued;
    } else {
      ptx::grid_dependency_wait();
      ptx::grid_launch_dependents();
    }
  } else {
    // ---- consumers: warp c reduces units c, c + 8, ...
    ptx::grid_dependency_wait();
    ptx::grid_launch_dependents();
    bool ok = ptx::mbar_wait_bounded(a_bar, 0u, abort_flag, kWaitBudgetNs);
    if (!ok && lane == 0) raise(kErrTimeoutMma);
    const uint4* av_all = reinterpret_cast<const uint4*>(smem + g.a_offset);
    for (int u = warp; ok && u < units; u += kRingConsumers) {
      const int s = u % g.stages;
      if (!ptx::mbar_wait_bounded(full(s), static_cast<uint32_t>(u / g.stages) & 1u, abort_flag, kWaitBudgetNs)) {
        if (lane == 0) raise(kErrTimeoutMma);
        break;
      }
      const int r = u / g.pieces;
      const int e0 = (u - r * g.pieces) * g.piece_elems;
      const int chunks = min(g.piece_elems, g.k - e0) >> 3;
      const uint4* wv = reinterpret_cast<const uint4*>(smem + static_cast<uint32_t>(s) * g.stage_bytes);
      const uint4* av = av_all + (e0 >> 3);
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 4
      for (int c = lane; c < chunks; c += 32) dot8<T>(wv[c], av[c], acc0, acc1);
      float acc = acc0 + acc1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      __syncwarp();
      if (lane == 0) {
        part[u] = acc;
        ptx::mbar_arrive(empty(s));
      }
    }
  }
  __syncthreads();
  const bool aborted = *abort_flag != 0;
  if (!aborted) {
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
      float sum = 0.0f;
      for (int pc = 0; pc < g.pieces; ++pc) sum += part[r * g.pieces + pc];
      const int row = row0 + r;
      const float b = g.epilogue != GLQ_EPILOGUE_NONE ? Vec<T>::to_f(static_cast<const T*>(g.bias)[row]) : 0.0f;
      static_cast<T*>(g.y)[row] = Vec<T>::from_f(apply_epilogue(sum, b, g.epilogue));
    }
  } else if (threadIdx.x == 0) {
    // Let this CTA's own bulk loads land before it exits.
    const int issued = *issued_slot;
    for (int u = max(0, issued - g.stages); u < issued; ++u) {
      if (!ptx::mbar_wait_bounded(full(u % g.stages), static_cast<uint32_t>(u / g.stages) & 1u, nullptr,
                                  kWaitBudgetNs)) {
        atomicOr(g.err, kErrTimeoutDrain);
        break;
      }
    }
  }
}

}  // namespace

namespace {

// Ring GEMV launch, or cudaErrorNotSupported when the shape does not fit it.
template <typename T>
cudaError_t launch_ring(const Problem& p, unsigned int* err, cudaStream_t s, int sm_count) {
  RingArgs g;
  g.a = p.a;
  g.w = p.b;
  g.ldw = p.b_ns;
  g.bias = p.bias;
  g.epilogue = p.epilogue;
  g.y = p.y;
  g.n = static_cast<int>(p.n);
  g.k = static_cast<int>(p.k);
  const int ctas = static_cast<int>(std::min<int64_t>(p.n, sm_count));
  g.rows_per_cta = static_cast<int>((p.n + ctas - 1) / ctas);
  const int grid = static_cast<int>((p.n + g.rows_per_cta - 1) / g.rows_per_cta);
  g.piece_elems = static_cast<int>(std::min<int64_t>(p.k, kRingPieceElems));
  g.pieces = static_cast<int>((p.k + g.piece_elems - 1) / g.piece_elems);
  g.stage_bytes = static_cast<uint32_t>(g.piece_elems) * 2u;
  const uint32_t a_bytes = static_cast<uint32_t>(p.k) * 2u;
  const uint32_t part_bytes = static_cast<uint32_t>(g.rows_per_cta * g.pieces) * 4u;
  const uint32_t fixed = a_bytes + ((part_bytes + 15u) & ~15u) + 1024u;
  if (!gemv_ring_fits(p.n, p.k, sm_count)) return cudaErrorNotSupported;
  g.stages = static_cast<int>(std::min<uint32_t>(kRingMaxStages, (kRingSmem - fixed) / g.stage_bytes));
  g.a_offset = static_cast<uint32_t>(g.stages) * g.stage_bytes;
  g.part_offset = g.a_offset + a_bytes;
  g.bar_offset = (g.part_offset + part_bytes + 15u) & ~15u;
  const uint32_t smem = g.bar_offset + static_cast<uint32_t>(2 * g.stages + 3) * 8u;
  g.err = err;
  g.flags = p.flags;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kRingThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (p.flags & GLQ_FLAG_NO_PDL) ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, gemv_ring_kernel<T>, g);
}

}  // namespace

cudaError_t gemv_prepare_device() {
  cudaError_t e = cudaFuncSetAttribute(gemv_ring_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kRingSmem));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemv_ring_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kRingSmem));
}

cudaError_t launch_gemv_ring(const Problem& p, unsigned int* err, cudaStream_t s, int sm_count) {
  if (p.dtype == GLQ_DTYPE_BF16) return launch_ring<__nv_bfloat16>(p, err, s, sm_count);
  return launch_ring<__half>(p, err, s, sm_count);
}

cudaError_t launch_gemv(const Problem& p, int split, unsigned int* /*err*/, cudaStream_t s) {
  GemvArgs g;
  g.a = p.a;
  g.w = p.b;
  g.ldw = p.b_ns;
  g.bias = p.bias;
  g.epilogue = p.epilogue;
  g.y = p.y;
  g.n = static_cast<int>(p.n);
  g.k = static_cast<int>(p.k);
  g.split = split;
  const int warps_per_row = split;
  int rows = (kBlockThreadsMax / 32) / warps_per_row;
  if (rows < 1) rows = 1;
  g.rows_per_block = rows;
  g.partial = p.partial;
  g.flags = p.flags;
  const size_t a_bytes = static_cast<size_t>(p.k / 8) * 16;
  g.a_in_smem = a_bytes <= kGemvSmemA ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((p.n + rows - 1) / rows), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(rows * warps_per_row * 32), 1, 1);
  cfg.dynamicSmemBytes = g.a_in_smem ? a_bytes : 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (p.flags & GLQ_FLAG_NO_PDL) ? 0 : 1;
  if (p.dtype == GLQ_DTYPE_BF16) return cudaLaunchKernelEx(&cfg, gemv_kernel<__nv_bfloat16, 8>, g);
  return cudaLaunchKernelEx(&cfg, gemv_kernel<__half, 8>, g);
}

}  // namespace glq
