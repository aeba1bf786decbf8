// glq_tc.cu -- tcgen05 linear kernel for sm_100a (M >= 2 tokens).
//
// Computes Y[m, n] = epilogue(sum_k A[m, k] * W[n, k]) for a K-contiguous
// weight W[N, K] (the lab's B = W^T view) and K-contiguous activations
// A[M, K], FP32 accumulation in tensor memory, one FP16/BF16 store.
//
// Design (swap-AB, decode shapes are weight-bandwidth bound):
//   * W rows fill the 128-lane MMA M dimension; the token batch is the MMA N
//     dimension (16..256), so M = 1..128 tokens cost one W pass.
//   * One CTA = 256 threads owns a 128- or 256-row W tile (one M = 128 MMA
//     and TMEM accumulator per 128 rows) x a token tile x one contiguous
//     range of 64-wide K blocks.  Thread 0 starts the TMA stream
//     (128-byte swizzle, K-major) into a STAGES-deep mbarrier ring before
//     anything else; warp 1 allocates TMEM and lane 0 issues tcgen05.mma; all
//     eight warps run the epilogue from TMEM (lane = W row, column = token),
//     two warps per 32-lane TMEM quarter splitting the token columns.
//   * Split-K: the K ranges of one tile are the CTAs of one thread-block
//     cluster.  After the main loop every CTA stages its FP32 partial tile in
//     its drained pipeline memory; lanes of warp 0 ship each other owner's
//     4-token groups with one DSMEM bulk copy each (rotated owner order),
//     completing on the owner's receive mbarrier; the owner reads its own
//     groups in place, waits only on that barrier, sums the S partials in
//     split order 0..S-1, applies bias + SiLU and stores.  The merge order is
//     fixed, so results are bitwise reproducible, and the only spin-waits are
//     bounded mbarrier waits.
//   * Prefill (M > 128): 256-token tiles launched token-tile-fastest (the
//     resident CTAs share W tiles); 256 x 256 output tiles when they fill a
//     wave.
//   * GATHER: the column-parallel layer's all-gather runs in the epilogue
//     (every rank's output over NVLink, then a bounded epoch handshake);
//     see the completion block at the end of the kernel.
//   * Programmatic dependent launch: every thread waits for the predecessor
//     grid (griddepcontrol.wait) before touching global memory and then lets
//     the next grid launch, so back-to-back calls overlap launch latency,
//     barrier set-up and TMEM allocation with the predecessor's tail.  With
//     GLQ_FLAG_STATIC_WEIGHTS the first W stages are requested before the
//     wait.
//   * W layouts: K-contiguous W [N, K] (a linear layer's weight) is loaded as
//     one 64(k) x TN box per stage and described K-major; the lab's own
//     B = [K, N] row-major (N contiguous) is loaded as TN/64 boxes of
//     64(n) x 64(k) and described MN-major to the MMA (WMN = true).  Both
//     land 128-byte swizzled; only the descriptors and the box shape differ.
//   * Every mbarrier wait is bounded (glq_ptx.cuh); on expiry the CTA raises
//     a bit in the device error word, stops issuing work, drains its own
//     in-flight TMA loads (bounded), still takes part in both cluster
//     barrier phases, frees TMEM and returns.
//
// Reference counterpart: ptx_mma_pipelined_kernel<..., SPLIT_K> +
// ptx_mma_splitk_reduce_kernel (csrc/ptx_mma.cuh:502-770, 851-868) and the
// Triton _matmul_kernel / _matmul_bias_silu_kernel / _splitk_* kernels
// (kernels.py:73-129, 191-249, 324-393), which compute the same sums with
// B = [K, N] operands on sm_80+ mma.sync.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "glq_internal.h"
#include "glq_ptx.cuh"

namespace glq {
namespace {

template <typename T>
struct Elem;

template <>
struct Elem<__half> {
  static constexpr int kFormat = 0;
  static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  __device__ static float to_f(__half v) { return __half2float(v); }
  __device__ static __half from_f(float v) { return __float2half_rn(v); }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kFormat = 1;
  static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  __device__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float apply_epilogue(float acc, float bias, int epilogue) {
  if (epilogue == GLQ_EPILOGUE_NONE) return acc;
  const float v = acc + bias;
  if (epilogue == GLQ_EPILOGUE_BIAS) return v;
  return __fdividef(v, 1.0f + __expf(-v));  // SiLU = v * sigmoid(v)
}

// One output element to every output buffer of the call (this rank's own Y,
// and with a fused gather every peer's Y over NVLink), starting with a
// different buffer per tile so the peers' links are loaded evenly.
template <typename T, typename Args>
__device__ __forceinline__ void store_out(const Args& args, long long offset, T v, int first) {
  for (int i = 0; i < args.n_out; ++i) {
    int o = first + i;
    if (o >= args.n_out) o -= args.n_out;
    static_cast<T*>(args.y_out[o])[offset] = v;
  }
}

constexpr int kTileK = 64;  // K elements per stage: one 128-byte swizzle row
constexpr uint32_t kMnBoxBytes = 64u * kTileK * 2u;  // one 64(n) x 64(k) MN-major W box
constexpr int kThreads = 256;
constexpr uint32_t kSmemLimit = 232448;  // 227 KB opt-in per CTA
// Two CTAs per SM: 228 KB of shared memory per SM, 1 KB reserved per block.
constexpr uint32_t kPairSmemBudget = 233472u / 2u - 1024u;

// BT: token tile (MMA N).  TN: W rows per CTA, one M = 128 MMA (and one TMEM
// accumulator of BT columns) per 128 rows.  A 256-row tile moves W in 32 KB
// TMA boxes, which streams HBM measurably better than 16 KB boxes at equal
// bytes in flight.  STAGES: depth of the TMA ring; 4 stages of a small token
// tile plus the split-K receive buffer keep a CTA under 113 KB of shared
// memory, so two CTAs share an SM.
template <int BT, int TN, int STAGES>
struct TcConfig {
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N for M=128 is 16..256 step 16");
  static_assert(TN == 128 || TN == 256, "tile rows are one or two M=128 MMAs");
  static constexpr int kAcc = TN / 128;
  static constexpr uint32_t kWTileBytes = TN * kTileK * 2;
  static constexpr uint32_t kATileBytes = BT * kTileK * 2;
  static constexpr uint32_t kStageBytes = kWTileBytes + kATileBytes;
  static constexpr int kStages = STAGES;
  static constexpr uint32_t kAccCols = kAcc * BT;
  static constexpr uint32_t kTmemCols =
      kAccCols <= 32 ? 32 : (kAccCols <= 64 ? 64 : (kAccCols <= 128 ? 128 : (kAccCols <= 256 ? 256 : 512)));
  static constexpr uint32_t kPipeBytes = kStages * kStageBytes;
  static constexpr uint32_t kBarrierBytes = (2 * kStages + 2) * 8 + 16;
  static_assert(kStageBytes % 1024 == 0, "stage bases must stay 1024-B aligned");
  static_assert(1024 + kPipeBytes + kBarrierBytes <= kSmemLimit, "pipeline exceeds shared memory");
};

struct TcArgs {
  int m, n, k;
  int num_kb;
  int split;
  int epilogue;
  const void* bias;
  void* y_out[GLQ_MAX_RANKS];  // output bases (this rank's columns); [0] alone unless gathering
  int n_out;
  long long ldy;
  float* partial;
  unsigned int* err;
  // Fused gather completion (counter == nullptr: plain call).
  unsigned long long* sig_out[GLQ_MAX_RANKS];  // every rank's signal slots
  unsigned long long* sig_in;                  // this rank's signal slots
  unsigned int* counter;
  unsigned long long epoch;
  int rank;
  uint32_t ys_offset;  // fused gather: FP16 output tile staging (bytes from the aligned base); ~0u = none
  int bulk_out;        // fused gather: staged rows leave by bulk copies (N % 8 == 0)
  uint32_t recv_offset;     // split-K receive buffer, bytes from the 1024-aligned base
  uint32_t stage_offset;    // split-K send staging buffer (inside the drained pipeline)
  int recv_overlaps;        // 1: the receive buffer reuses the drained pipeline stages
  uint32_t barrier_offset;  // mbarriers, bytes from the aligned base
  unsigned int flags;       // glq_flags
  // LDG kernels: W [N, K] K-contiguous rows that TMA cannot address (row
  // pitch or base not 16-byte aligned), loaded by the SM.
  const void* w_ptr;
  long long w_pitch_bytes;
};

// W rows loaded by the SM instead of TMA: warps 2..5 fill each stage.
constexpr int kLdgWarps = 4;
constexpr int kLdgThreads = kLdgWarps * 32;

// ---- W producer for rows that TMA cannot address (LDG kernels).
//
// Thread t (0..127, warps 2..5) owns 16-byte chunk c = t % 8 of rows
// r = t / 8 + 16 j (j = 0..7) of each 128-row x 64-K stage, so a warp covers
// four rows of 128 contiguous bytes per step.  Chunk c of a row starts at
// byte offset `shift` (the same for every chunk of the row) inside the
// aligned granule G + 16 c; its bytes are that granule and the next one,
// which is the neighbouring lane's granule (shuffle) except for c = 7, which
// loads it.  A granule is read only if it holds bytes of the row (the first
// always does unless the row is past N; the others are skipped past the
// row's end), and an aligned 16-byte granule never crosses a page.  Columns
// k >= K and rows n >= N are written as zero, as TMA's out-of-bounds fill
// would.  Each chunk goes to its 128-byte-swizzle position (chunk c of row r
// at r * 128 + ((c ^ (r % 8)) * 16)), the layout the K-major UMMA descriptor
// reads; the writes are made visible to the tensor core with
// fence.proxy.async before every thread's arrival on the stage's full
// barrier.  All loads of a half stage are issued before any is used.
template <typename T, int BT, int TN, int STAGES, typename FullBar, typename EmptyBar, typename Raise>
__device__ __forceinline__ void ldg_fill_w(const TcArgs& args, uint8_t* smem, int kb_begin, int nkb, int tile_n,
                                           FullBar full_bar, EmptyBar empty_bar, const volatile int* abort_flag,
                                           Raise raise) {
  using Cfg = TcConfig<BT, TN, STAGES>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kRowsPerPass = kLdgThreads / 8;  // 16
  constexpr int kPasses = TN / kRowsPerPass;      // 8
  constexpr int kBatch = 4;                       // passes whose loads are in flight together
  const int t = static_cast<int>(threadIdx.x) - 64;
  const int lane = t & 31;
  const int c = t & 7;
  const uintptr_t wbase = reinterpret_cast<uintptr_t>(args.w_ptr);
  const long long row_bytes = static_cast<long long>(args.k) * 2;
  for (int i = 0; i < nkb; ++i) {
    const int stage = i % kStages;
    if (i >= kStages) {
      bool ok = true;
      if (lane == 0) {
        ok = ptx::mbar_wait_bounded(empty_bar(stage), static_cast<uint32_t>(i / kStages - 1) & 1u, abort_flag,
                                    kWaitBudgetNs);
      }
      if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) {
        if (lane == 0) raise(kErrTimeoutProducer);
        return;
      }
    }
    const long long k0 = static_cast<long long>(kb_begin + i) * kTileK;
    uint8_t* const w_stage = smem + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
#pragma unroll
    for (int b = 0; b < kPasses; b += kBatch) {
      uint4 lo[kBatch], hi[kBatch];
      unsigned shift[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int r = t / 8 + kRowsPerPass * (b + j);
        const long long n = static_cast<long long>(tile_n) * TN + r;
        lo[j] = make_uint4(0u, 0u, 0u, 0u);
        hi[j] = make_uint4(0u, 0u, 0u, 0u);
        shift[j] = 0;
        if (n < args.n) {
          const uintptr_t row_begin = wbase + static_cast<uintptr_t>(n * args.w_pitch_bytes);
          const uintptr_t row_end = row_begin + static_cast<uintptr_t>(row_bytes);
          const uintptr_t first = row_begin + static_cast<uintptr_t>(k0 * 2);
          const uintptr_t g = (first & ~static_cast<uintptr_t>(15)) + 16u * static_cast<uintptr_t>(c);
          shift[j] = static_cast<unsigned>(first & 15u);
          if (g < row_end) lo[j] = __ldg(reinterpret_cast<const uint4*>(g));
          if (c == 7 && shift[j] != 0 && g + 16 < row_end) hi[j] = __ldg(reinterpret_cast<const uint4*>(g + 16));
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const uint32_t nx = __shfl_down_sync(0xffffffffu, lo[j].x, 1);
        const uint32_t ny = __shfl_down_sync(0xffffffffu, lo[j].y, 1);
        const uint32_t nz = __shfl_down_sync(0xffffffffu, lo[j].z, 1);
        const uint32_t nw = __shfl_down_sync(0xffffffffu, lo[j].w, 1);
        if (c != 7) hi[j] = make_uint4(nx, ny, nz, nw);
        const int r = t / 8 + kRowsPerPass * (b + j);
        const long long n = static_cast<long long>(tile_n) * TN + r;
        const long long valid = static_cast<long long>(args.k) - (k0 + 8 * c);
        uint32_t out[4] = {0u, 0u, 0u, 0u};
        if (n < args.n && valid > 0) {
          const uint32_t w[8] = {lo[j].x, lo[j].y, lo[j].z, lo[j].w, hi[j].x, hi[j].y, hi[j].z, hi[j].w};
          const unsigned q = shift[j] >> 2;
          const unsigned bits = (shift[j] & 3u) * 8u;
          uint32_t pick[5];
#pragma unroll
          for (int e = 0; e < 5; ++e) {
            const uint32_t x0 = w[e], x1 = w[e + 1 < 8 ? e + 1 : 7], x2 = w[e + 2 < 8 ? e + 2 : 7],
                           x3 = w[e + 3 < 8 ? e + 3 : 7];
            pick[e] = q == 0 ? x0 : q == 1 ? x1 : q == 2 ? x2 : x3;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) out[e] = __funnelshift_r(pick[e], pick[e + 1], bits);
          if (valid < 8) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (2 * e >= valid) {
                out[e] = 0u;
              } else if (2 * e + 1 >= valid) {
                out[e] &= 0xFFFFu;
              }
            }
          }
        }
        *reinterpret_cast<uint4*>(w_stage + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive(full_bar(stage));
  }
}

// LDG: the W tiles are written into the swizzled stages by warps 2..5 from
// plain 16-byte loads (K-major W, 128-row tiles, no gather); two CTAs per SM
// must still fit, so these instantiations are capped at 128 registers.
template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, bool LDG = false>
__global__ void __launch_bounds__(kThreads, LDG ? 2 : 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_a, const TcArgs args) {
  static_assert(!LDG || (!WMN && !GATHER && TN == 128), "SM-loaded W: K-major 128-row tiles only");
  using Cfg = TcConfig<BT, TN, STAGES>;
  constexpr uint32_t kWTileBytes = Cfg::kWTileBytes;
  constexpr int kStages = Cfg::kStages;

  extern __shared__ uint8_t smem_dyn[];
  const uint32_t raw_base = ptx::smem_addr(smem_dyn);
  const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
  uint8_t* smem = smem_dyn + pad;
  const uint32_t sbase = raw_base + pad;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + args.barrier_offset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_slot = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = args.split;
  const int s = blockIdx.x;  // split index == CTA rank in the (split,1,1) cluster
  // Token tiles vary fastest in launch order, so the CTAs resident at one
  // time share W tiles (read from HBM once) and re-read the smaller A from L2.
  const int tile_t = blockIdx.y;
  const int tile_n = blockIdx.z;
  const int kb_begin = static_cast<int>((static_cast<long long>(s) * args.num_kb) / split);
  const int kb_end = static_cast<int>((static_cast<long long>(s + 1) * args.num_kb) / split);
  const int nkb = kb_end - kb_begin;

  auto full_bar = [&](int i) { return ptx::smem_addr(&bars[i]); };
  auto empty_bar = [&](int i) { return ptx::smem_addr(&bars[kStages + i]); };
  const uint32_t done_bar = ptx::smem_addr(&bars[2 * kStages]);
  const uint32_t recv_bar = ptx::smem_addr(&bars[2 * kStages + 1]);

  // Token columns of this tile and, for split-K, the 4-column groups this
  // CTA owns: groups are dealt to the S ranks as [r*G/S, (r+1)*G/S).
  const long long m0 = static_cast<long long>(tile_t) * BT;
  const int mr = static_cast<int>(min(static_cast<long long>(BT), args.m - m0));
  const int groups = (mr + 3) >> 2;
  const int own_lo = (s * groups) / split;
  const int own_hi = ((s + 1) * groups) / split;
  const int own_width = own_hi - own_lo;
  auto raise = [&](unsigned int bit) {
    atomicOr(args.err, bit);
    *abort_flag = 1;
  };

  // ---- TMA producer state (thread 0): W streamed once (evict-first), A reused (evict-last).
  uint64_t pol_w = 0, pol_a = 0;
  int issued = 0;
  // Stage i: one expect_tx for the whole stage, then the W tile and the A tile.
  auto issue_w = [&](int i) {
    const int stage = i % kStages;
    const uint32_t w_dst = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
    ptx::mbar_arrive_expect_tx(full_bar(stage), Cfg::kStageBytes);
    if constexpr (WMN) {
      // TN/64 boxes of 64 N-contiguous W rows x 64 K rows, 8 KB apart.
#pragma unroll
      for (int j = 0; j < TN / 64; ++j) {
        ptx::tma_load_2d(w_dst + static_cast<uint32_t>(j) * kMnBoxBytes, &tmap_w, tile_n * TN + 64 * j,
                         (kb_begin + i) * kTileK, full_bar(stage), pol_w);
      }
    } else {
      ptx::tma_load_2d(w_dst, &tmap_w, (kb_begin + i) * kTileK, tile_n * TN, full_bar(stage), pol_w);
    }
  };
  auto issue_a = [&](int i) {
    const int stage = i % kStages;
    const uint32_t a_dst = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes + kWTileBytes;
    ptx::tma_load_2d(a_dst, &tmap_a, (kb_begin + i) * kTileK, tile_t * BT, full_bar(stage), pol_a);
  };
  auto issue = [&](int i) {
    if constexpr (LDG) {
      // The W half of the stage arrives through the producer warps' arrivals.
      ptx::mbar_arrive_expect_tx(full_bar(i % kStages), Cfg::kATileBytes);
    } else {
      issue_w(i);
    }
    issue_a(i);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      // LDG: thread 0 (A, expect_tx) plus every W producer thread arrives.
      ptx::mbar_init(full_bar(i), LDG ? 1 + kLdgThreads : 1);
      ptx::mbar_init(empty_bar(i), 1);
    }
    ptx::mbar_init(done_bar, 1);
    ptx::mbar_init(recv_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    // The owner expects 16 bytes per (remote source rank, W row, owned
    // group); its own partial is read in place.
    if (split > 1) {
      ptx::mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(split - 1) * TN *
                                               static_cast<uint32_t>(own_width) * 16u);
    }
    ptx::prefetch_tensormap(&tmap_w);
    ptx::prefetch_tensormap(&tmap_a);
    pol_w = ptx::policy_evict_first();
    pol_a = ptx::policy_evict_last();
    // Start the stream before anything else: the first kStages stages are
    // free, so these loads need no wait.  With programmatic dependent launch
    // the predecessor kernel may still be running: A (and W unless the
    // caller declared the weights static) is read only after the dependency
    // wait.
    const int first = nkb < kStages ? nkb : kStages;
    const bool static_w = !LDG && (args.flags & GLQ_FLAG_STATIC_WEIGHTS) != 0;
    if (static_w) {
      for (int i = 0; i < first; ++i) issue_w(i);
    }
    ptx::grid_dependency_wait();
    for (; issued < first; ++issued) {
      if constexpr (LDG) {
        ptx::mbar_arrive_expect_tx(full_bar(issued), Cfg::kATileBytes);
      } else {
        if (!static_w) issue_w(issued);
      }
      issue_a(issued);
    }
    *issued_slot = issued;
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_d = *tmem_slot;
  // Every thread orders its own global accesses after the predecessor grid
  // (immediate once thread 0 has passed it), then lets the next grid launch.
  ptx::grid_dependency_wait();
  ptx::grid_launch_dependents();

  // Warp w reads TMEM lanes 32*(w%4)..+31.  With two accumulators warpgroup
  // h owns accumulator h (W rows 128h..) and all its columns; with one, the
  // two warpgroups take alternate 16-column chunks of it.
  const int lane_group = warp & 3;
  const int half = warp >> 2;
  const int acc_idx = Cfg::kAcc == 2 ? half : 0;
  const int q_first = Cfg::kAcc == 2 ? 0 : half;
  const int q_step = Cfg::kAcc == 2 ? 1 : 2;
  const int n_local = acc_idx * 128 + lane_group * 32 + lane;  // == threadIdx.x % TN
  const long long n = static_cast<long long>(tile_n) * TN + n_local;
  const bool n_ok = n < args.n;
  float bias_v = 0.0f;
  if (args.epilogue != GLQ_EPILOGUE_NONE && n_ok) {
    bias_v = Elem<T>::to_f(static_cast<const T*>(args.bias)[n]);
  }

  // Cluster barrier phase 1 proves every CTA of the cluster is running (its
  // receive barrier initialised) before anyone stores into it.  With a
  // dedicated receive buffer it is armed now and the epilogue warps absorb
  // the wait during the main loop; when the buffer reuses the pipeline it is
  // armed only after the main loop.
  const bool recv_dedicated = split > 1 && !args.recv_overlaps;
  // W producer warps (LDG) wait after their loop instead.
  const bool ldg_producer = LDG && warp >= 2 && warp < 2 + kLdgWarps;
  if (recv_dedicated) {
    ptx::cluster_arrive_relaxed();
    if (warp >= 2 && !ldg_producer) ptx::cluster_wait();
  }

  if (warp == 0) {
    if (lane == 0) {
      for (int i = issued; i < nkb; ++i) {
        const int stage = i % kStages;
        const uint32_t round = static_cast<uint32_t>(i / kStages);
        if (!ptx::mbar_wait_bounded(empty_bar(stage), (round - 1u) & 1u, abort_flag, kWaitBudgetNs)) {
          raise(kErrTimeoutProducer);
          break;
        }
        issue(i);
        issued = i + 1;
      }
      *issued_slot = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: per 128 W rows h, D_h[128 x BT] += W_h[128 x 64] * A[BT x 64]^T;
      // accumulator h occupies TMEM columns [h*BT, (h+1)*BT).
      constexpr uint32_t idesc = ptx::umma_idesc_f16(128, BT, Elem<T>::kFormat, WMN ? 1 : 0);
      // Descriptor start-address step (16-byte units) per K = 16 MMA: 32 B
      // along a K-major swizzled row, or 16 K rows of 128 B when MN-major.
      constexpr uint32_t kWStep = WMN ? 128u : 2u;
      for (int i = 0; i < nkb; ++i) {
        const int stage = i % kStages;
        const uint32_t round = static_cast<uint32_t>(i / kStages);
        if (!ptx::mbar_wait_bounded(full_bar(stage), round & 1u, abort_flag, kWaitBudgetNs)) {
          raise(kErrTimeoutMma);
          break;
        }
        ptx::tc_fence_after_sync();
        const uint32_t w_src = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
        const uint64_t w_desc = WMN ? ptx::umma_desc_mn_sw128(w_src) : ptx::umma_desc_k_sw128(w_src);
        const uint64_t a_desc = ptx::umma_desc_k_sw128(w_src + kWTileBytes);
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk) {
          // Each MMA consumes K = 16.  The 128-row halves of a 256-row W
          // tile are 16 KB (1024 units) apart in both layouts.
#pragma unroll
          for (int h = 0; h < Cfg::kAcc; ++h) {
            ptx::tc_mma_f16(tmem_d + static_cast<uint32_t>(h * BT), w_desc + 1024u * h + kWStep * kk,
                            a_desc + 2u * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        ptx::tc_commit(empty_bar(stage));
      }
      ptx::tc_commit(done_bar);
    }
  } else if (ldg_producer) {
    if constexpr (LDG) ldg_fill_w<T, BT, TN, STAGES>(args, smem, kb_begin, nkb, tile_n, full_bar, empty_bar,
                                                      abort_flag, raise);
  }
  __syncwarp();
  if (recv_dedicated && (warp < 2 || ldg_producer)) ptx::cluster_wait();

  // ---- Epilogue: 8 warps (rows and chunks as assigned above).
  if (!ptx::mbar_wait_bounded(done_bar, 0u, abort_flag, kWaitBudgetNs)) {
    raise(kErrTimeoutEpilogue);
  }
  __syncthreads();
  const bool aborted = *abort_flag != 0;
  ptx::tc_fence_after_sync();

  const int chunks = (mr + 15) >> 4;
  // Output stores: this rank's Y directly; with a fused gather the FP16
  // tile is first staged in shared memory as [token][W row] (the drained
  // pipeline), then written to every rank's Y as 16-byte vectors (one
  // NVLink-friendly store per 8 outputs instead of eight 2-byte ones).
  T* const y = static_cast<T*>(args.y_out[0]);
  const int out_first = GATHER ? static_cast<int>((blockIdx.y + blockIdx.z) % static_cast<unsigned>(args.n_out)) : 0;
  const bool gather_staged = GATHER && args.ys_offset != ~0u;
  T* const ys = reinterpret_cast<T*>(smem + (gather_staged ? args.ys_offset : 0u));
  // mm: token within this CTA's token tile; mm_base: first token of the staged rows.
  auto store = [&](int mm, int mm_base, T v) {
    if constexpr (GATHER) {
      if (gather_staged) {
        ys[(mm - mm_base) * TN + n_local] = v;
      } else {
        store_out<T>(args, (m0 + mm) * args.ldy + n, v, out_first);
      }
    } else {
      y[(m0 + mm) * args.ldy + n] = v;
    }
  };
  // Staged rows [mm_base, mm_base + rows) of the tile to every output.
  auto flush_staged = [&](int mm_base, int rows) {
    if constexpr (GATHER) {
      if (!gather_staged) return;
      const long long n_tile = static_cast<long long>(tile_n) * TN;
      if (args.bulk_out) {
        // One TMA-engine copy per (token row, rank): 256-byte NVLink writes
        // instead of 16-byte stores from the SM.
        ptx::fence_proxy_async_smem();
        __syncthreads();
        if (warp == 0) {
          const long long valid = min(static_cast<long long>(TN), static_cast<long long>(args.n) - n_tile);
          const uint32_t bytes = static_cast<uint32_t>(valid) * static_cast<uint32_t>(sizeof(T));
          for (int idx = lane; valid > 0 && idx < rows * args.n_out; idx += 32) {
            const int row = idx / args.n_out;
            int o = out_first + (idx - row * args.n_out);
            if (o >= args.n_out) o -= args.n_out;
            ptx::bulk_store_1d(static_cast<T*>(args.y_out[o]) + (m0 + mm_base + row) * args.ldy + n_tile,
                               ptx::smem_addr(ys + row * TN), bytes);
          }
          ptx::bulk_commit();
          ptx::bulk_wait_all();
          ptx::fence_proxy_async_global();
        }
        return;
      }
      __syncthreads();
      constexpr int kVec = 8;                // FP16/BF16 outputs per 16-byte store
      constexpr int kChunks = TN / kVec;
      for (int idx = threadIdx.x; idx < rows * kChunks; idx += kThreads) {
        const int row = idx / kChunks;
        const int c = idx - row * kChunks;
        const long long n0 = n_tile + c * kVec;
        const long long off = (m0 + mm_base + row) * args.ldy + n0;
        const T* src = ys + row * TN + c * kVec;
        if (n0 + kVec <= args.n) {
          const uint4 v = *reinterpret_cast<const uint4*>(src);
          for (int i = 0; i < args.n_out; ++i) {
            int o = out_first + i;
            if (o >= args.n_out) o -= args.n_out;
            *reinterpret_cast<uint4*>(static_cast<T*>(args.y_out[o]) + off) = v;
          }
        } else {
          for (int e = 0; e < kVec && n0 + e < args.n; ++e) store_out<T>(args, off + e, src[e], out_first);
        }
      }
    }
  };
  const uint32_t t_row =
      tmem_d + (static_cast<uint32_t>(lane_group * 32) << 16) + static_cast<uint32_t>(acc_idx * BT);

  if (split == 1) {
    if (!aborted) {
      for (int q = q_first; q < chunks; q += q_step) {
        uint32_t r[16];
        ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(q * 16), r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int mm = q * 16 + j;
          if (mm < mr && n_ok) {
            store(mm, 0, Elem<T>::from_f(apply_epilogue(__uint_as_float(r[j]), bias_v, args.epilogue)));
          }
        }
      }
    }
    flush_staged(0, aborted ? 0 : mr);
  } else {
    // Split-K merge.  Every CTA stages its FP32 partial tile in its own
    // drained pipeline memory as [group][row] (16 bytes per entry, so
    // consecutive rows are consecutive: no bank conflicts).  4-token groups
    // are dealt to the S ranks as [r*G/S, (r+1)*G/S), so the groups of rank r
    // form one contiguous block; lane (r - s) mod S of warp 0 ships it to
    // rank r's receive slot for source s with one bulk copy that completes
    // its bytes on rank r's receive barrier.  Each owner waits only on that
    // barrier, then sums the S partials of its groups in split order 0..S-1
    // (its own from its staging buffer), applies bias + SiLU and stores.
    const uint32_t recv = sbase + args.recv_offset;
    const uint32_t stage_out = sbase + args.stage_offset;
    if (!recv_dedicated) {
      ptx::cluster_arrive_relaxed();  // this CTA's pipeline is drained
      ptx::cluster_wait();
    }
    if (!aborted) {
      for (int q = q_first; q < chunks; q += q_step) {
        uint32_t r[16];
        ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(q * 16), r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int g = 4 * q + h;
          if (g < groups) {
            // [group][row]: consecutive threads (rows) write consecutive 16 B.
            uint4* dst = reinterpret_cast<uint4*>(smem + args.stage_offset) + (g * TN + n_local);
            *dst = make_uint4(r[4 * h], r[4 * h + 1], r[4 * h + 2], r[4 * h + 3]);
          }
        }
        if (args.partial != nullptr && n_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int mm = q * 16 + j;
            if (mm < mr) {
              args.partial[(static_cast<long long>(s) * args.m + m0 + mm) * args.n + n] =
                  __uint_as_float(r[j]);
            }
          }
        }
      }
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();
    // Lane d of warp 0 ships this rank's groups of owner (s + d) % split, so
    // the copies enter the engine together and every owner is fed by a
    // different source at any moment.
    if (warp == 0 && lane >= 1 && lane < split && !aborted) {
      const int owner = (s + lane) % split;
      const int g_lo = (owner * groups) / split;
      const int width = ((owner + 1) * groups) / split - g_lo;
      if (width > 0) {
        const uint32_t bytes = static_cast<uint32_t>(TN * width) * 16u;
        // Owner's receive slot for source s: the S - 1 remote sources in rank order.
        const uint32_t slot = static_cast<uint32_t>(s < owner ? s : s - 1);
        ptx::bulk_copy_to_peer(ptx::map_to_rank(recv + slot * bytes, static_cast<uint32_t>(owner)),
                               stage_out + static_cast<uint32_t>(g_lo * TN) * 16u, bytes,
                               ptx::map_to_rank(recv_bar, static_cast<uint32_t>(owner)));
      }
    }
    const bool received = ptx::mbar_wait_bounded(recv_bar, 0u, aborted ? abort_flag : nullptr, kWaitBudgetNs);
    if (!received && !aborted) raise(kErrTimeoutEpilogue);
    // Phase 2: a CTA arrives once its own receive barrier has completed, so
    // passing the wait (after the stores below) means every copy of the
    // cluster has landed and no CTA leaves while a copy from or to it is in
    // flight.  Relaxed: the barrier orders nothing else (the receive barrier
    // already did).
    ptx::cluster_arrive_relaxed();
    if (received && !aborted) {
      const float4* rv = reinterpret_cast<const float4*>(smem + args.recv_offset);
      const float4* own = reinterpret_cast<const float4*>(smem + args.stage_offset) + own_lo * TN;
      // Thread t reduces W row t % TN (its epilogue row) for owned groups
      // j = t / TN, t / TN + 256 / TN, ...; this rank's own partial is read
      // from its staging buffer, the others from the receive slots.
      for (int j = threadIdx.x / TN; j < own_width; j += kThreads / TN) {
        // All loads first (independent), then the sum in split order.
        float4 part[GLQ_MAX_SPLIT];
#pragma unroll
        for (int src = 0; src < GLQ_MAX_SPLIT; ++src) {
          if (src < split) {
            const int slot = src < s ? src : src - 1;
            part[src] = src == s ? own[j * TN + n_local] : rv[(slot * own_width + j) * TN + n_local];
          }
        }
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int src = 0; src < GLQ_MAX_SPLIT; ++src) {
          if (src < split) {
            acc.x += part[src].x;
            acc.y += part[src].y;
            acc.z += part[src].z;
            acc.w += part[src].w;
          }
        }
        const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
        const int mm0 = 4 * (own_lo + j);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int mm = mm0 + c;
          if (mm < mr && n_ok) {
            store(mm, 4 * own_lo, Elem<T>::from_f(apply_epilogue(vals[c], bias_v, args.epilogue)));
          }
        }
      }
    }
    flush_staged(4 * own_lo, (received && !aborted) ? max(0, min(4 * own_width, mr - 4 * own_lo)) : 0);
    ptx::cluster_wait();
  }

  // ---- Teardown: after an abort, let this CTA's own TMA loads land first.
  if (aborted && threadIdx.x == 0) {
    const int done_issue = *issued_slot;
    for (int i = max(0, done_issue - kStages); i < done_issue; ++i) {
      if (!ptx::mbar_wait_bounded(full_bar(i % kStages), static_cast<uint32_t>(i / kStages) & 1u,
                                  nullptr, kWaitBudgetNs)) {
        atomicOr(args.err, kErrTimeoutDrain);
        break;
      }
    }
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc(tmem_d, Cfg::kTmemCols);
  }

  // ---- Fused gather completion.  The output tile left as 16-byte stores
  // (generic proxy) to this rank's Y and over NVLink to every peer's.  After
  // the CTA barrier, thread 0 fences at GPU scope (cumulative over the CTA's
  // stores, local and peer) and counts the CTA in with an acq_rel atomic
  // add; the CTA whose add completes the count synchronises with every other
  // CTA's release on this GPU, resets the counter, fences at system scope (so
  // every CTA's stores precede, in causality order, what follows), writes the
  // epoch into this rank's slot of every rank's signal array and waits,
  // bounded, until every rank has written its slot here, one lane per rank
  // reading the slots with system-scope acquire loads (which order the
  // peers' slices before the kernel's end).  Only that one CTA pays a
  // system-scope fence (hundreds of concurrent ones serialise), and no CTA
  // waits for its NVLink writes to land before counting in.  The kernel
  // completes only when this rank's output holds all slices.  Every wait is
  // bounded; on expiry the device error word gets kErrTimeoutPeer and the
  // kernel returns.
  if constexpr (GATHER) {
    __syncthreads();
    bool last = false;
    if (threadIdx.x == 0) {
      // This CTA's output stores (every thread's, local and over NVLink,
      // ordered before by the barrier) are released at GPU scope with the
      // count; the CTA whose increment completes the count is the last and
      // publishes for the grid.
      ptx::fence_acq_rel_gpu();
      const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
      last = ptx::atom_add_acq_rel_gpu(args.counter, 1u) == total - 1u;
    }
    if (warp == 0) {
      last = __shfl_sync(0xffffffffu, last ? 1 : 0, 0) != 0;
      if (last) {
        if (lane == 0) {
          *args.counter = 0u;  // every CTA of this grid has counted in
          // The one system-scope fence of the grid: cumulative over every
          // CTA's stores synchronised above, so they are visible to any
          // rank that sees the epoch written after it.
          ptx::fence_acq_rel_sys();
          for (int r = 0; r < args.n_out; ++r) ptx::st_relaxed_sys_u64(args.sig_out[r] + args.rank, args.epoch);
        }
        __syncwarp();
        // Lane r waits for rank r's epoch (all ranks' slots polled at once).
        const uint64_t t0 = ptx::globaltimer_ns();
        uint32_t polls = 0;
        bool ok = true;
        if (lane < args.n_out) {
          while (ptx::ld_acquire_sys_u64(args.sig_in + lane) < args.epoch) {
            if ((++polls & 63u) == 0u && (ptx::globaltimer_ns() - t0 > kWaitBudgetNs || polls > (1u << 26))) {
              ok = false;
              break;
            }
          }
        }
        const bool all_ok = __all_sync(0xffffffffu, ok);
        if (lane == 0 && !all_ok) atomicOr(args.err, kErrTimeoutPeer);
      }
    }
  }
}

// ------------------------------------------------------------------ host

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode;
}

// 2-D map of a row-major matrix rows x cols (cols contiguous) with a row
// pitch in bytes; box box_rows x box_cols, 128-byte swizzle, OOB zero fill.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, int64_t cols, int64_t rows,
               int64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_pitch_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, bool LDG = false>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(tc_linear_kernel<T, BT, TN, STAGES, WMN, GATHER, LDG>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
}

template <typename T, int BT, int TN, int STAGES>
cudaError_t set_attrs() {
  cudaError_t e;
  if constexpr (TN == 128) {
    if ((e = set_attr<T, BT, TN, STAGES, false, false, true>()) != cudaSuccess) return e;
  }
  if ((e = set_attr<T, BT, TN, STAGES, false, false>()) != cudaSuccess) return e;
  if ((e = set_attr<T, BT, TN, STAGES, true, false>()) != cudaSuccess) return e;
  if ((e = set_attr<T, BT, TN, STAGES, false, true>()) != cudaSuccess) return e;
  return set_attr<T, BT, TN, STAGES, true, true>();
}

template <typename T>
cudaError_t set_attrs_all() {
  cudaError_t e;
  if ((e = set_attrs<T, 16, 256, 4>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 32, 256, 4>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 256, 256, 3>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 16, 128, kPairStages>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 32, 128, kPairStages>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 16, 128, 8>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 32, 128, 8>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 64, 128, 8>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 128, 128, 6>()) != cudaSuccess) return e;
  return set_attrs<T, 256, 128, 4>();
}

template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, bool LDG = false>
cudaError_t launch_typed(const Problem& p, int split, const Gather* g, unsigned int* err, cudaStream_t stream) {
  constexpr int64_t esz = 2;
  CUtensorMap tmap_w, tmap_a;
  const int64_t a_pitch = p.m > 1 ? p.a_rs * esz : ((p.k * esz + 15) / 16) * 16;
  bool ok = true;
  if constexpr (LDG) {
    // W is read by the SM: no W tensor map (the kernel gets A's as a stand-in).
  } else if constexpr (WMN) {
    // B = [K, N]: rows k (pitch b_ks), N contiguous; boxes 64(n) x 64(k).
    ok = encode_2d(&tmap_w, Elem<T>::kTmaType, p.b, p.n, p.k, p.b_ks * esz, 64, kTileK);
  } else {
    // W = B^T: rows n (pitch b_ns), K contiguous; boxes 64(k) x TN.
    const int64_t w_pitch = p.n > 1 ? p.b_ns * esz : ((p.k * esz + 15) / 16) * 16;
    ok = encode_2d(&tmap_w, Elem<T>::kTmaType, p.b, p.k, p.n, w_pitch, kTileK, TN);
  }
  // A: rows m (pitch a_rs), K contiguous; boxes 64(k) x BT.
  if (!ok || !encode_2d(&tmap_a, Elem<T>::kTmaType, p.a, p.k, p.m, a_pitch, kTileK, BT)) {
    return cudaErrorInvalidValue;
  }
  if constexpr (LDG) tmap_w = tmap_a;
  using Cfg = TcConfig<BT, TN, STAGES>;
  TcArgs args;
  args.m = static_cast<int>(p.m);
  args.n = static_cast<int>(p.n);
  args.k = static_cast<int>(p.k);
  args.num_kb = static_cast<int>(tc_k_blocks(p.k));
  args.split = split;
  args.epilogue = p.epilogue;
  args.bias = p.bias;
  args.n_out = 1;
  args.y_out[0] = p.y;
  args.counter = nullptr;
  args.sig_in = nullptr;
  args.epoch = 0;
  args.rank = 0;
  for (int r = 0; r < GLQ_MAX_RANKS; ++r) args.sig_out[r] = nullptr;
  if (g != nullptr) {
    args.n_out = g->world;
    for (int r = 0; r < g->world; ++r) {
      args.y_out[r] = g->y[r];
      args.sig_out[r] = g->signal[r];
    }
    args.sig_in = g->signal[g->rank];
    args.counter = g->counter;
    args.epoch = g->epoch;
    args.rank = g->rank;
  }
  args.ldy = p.ldy;
  args.partial = p.partial;
  args.err = err;
  args.flags = p.flags;
  args.w_ptr = LDG ? p.b : nullptr;
  args.w_pitch_bytes = LDG && p.n > 1 ? p.b_ns * esz : 0;
  // Shared memory: [pipeline stages][split-K receive buffer][mbarriers].
  // The receive buffer ((split - 1) remote sources x TN rows x owned groups
  // x 16 B) gets its own
  // region when it fits; otherwise it reuses the drained stages, after one
  // more cluster barrier.  The send staging buffer (TN rows x all groups x
  // 16 B) always reuses the drained stages, after the receive buffer.
  uint32_t recv_bytes = 0, stage_bytes = 0;
  if (split > 1) {
    const uint32_t groups = BT / 4;
    const uint32_t width = (groups + split - 1) / split;
    recv_bytes = static_cast<uint32_t>(split - 1) * TN * width * 16u;
    stage_bytes = TN * groups * 16u;
  }
  // The two-CTAs-per-SM configuration keeps under half an SM.
  constexpr bool kPair = TN == 128 && BT <= 32 && STAGES == kPairStages;
  const uint32_t budget = kPair ? kPairSmemBudget : kSmemLimit;
  const bool dedicated = 1024 + Cfg::kPipeBytes + recv_bytes + Cfg::kBarrierBytes <= budget;
  args.recv_offset = dedicated ? Cfg::kPipeBytes : 0;
  args.stage_offset = dedicated ? 0 : ((recv_bytes + 1023u) & ~1023u);
  args.recv_overlaps = dedicated ? 0 : 1;
  if (args.stage_offset + stage_bytes > Cfg::kPipeBytes) return cudaErrorInvalidValue;
  // Fused gather: the FP16 output tile is staged in the drained pipeline,
  // after the split-K buffers (16-byte rows need 16-byte aligned outputs).
  args.ys_offset = ~0u;
  if (GATHER && (p.ldy * esz) % 16 == 0 && g != nullptr) {
    bool bases_ok = true;
    for (int r = 0; r < g->world; ++r) bases_ok = bases_ok && (reinterpret_cast<uintptr_t>(g->y[r]) % 16 == 0);
    const uint32_t used = split > 1 ? (dedicated ? stage_bytes : args.stage_offset + stage_bytes) : 0u;
    const uint32_t ys_off = (used + 15u) & ~15u;
    const uint32_t rows = split > 1 ? 4u * ((BT / 4 + split - 1) / split) : static_cast<uint32_t>(BT);
    if (bases_ok && ys_off + rows * TN * static_cast<uint32_t>(esz) <= Cfg::kPipeBytes) args.ys_offset = ys_off;
  }
  // Bulk copies need 16-byte row segments: every tile's valid width a multiple of 8.
  // Outputs leave by 16-byte stores from all threads (generic proxy): the
  // grid's single system-scope fence then covers them, where bulk copies
  // (async proxy) had to be awaited by every CTA before it could count in.
  args.bulk_out = 0;
  const uint32_t body = dedicated ? Cfg::kPipeBytes + recv_bytes : Cfg::kPipeBytes;
  args.barrier_offset = (body + 15u) & ~15u;
  const uint32_t smem_bytes = 1024 + args.barrier_offset + Cfg::kBarrierBytes;
  if (smem_bytes > budget) return cudaErrorInvalidValue;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(split), static_cast<unsigned>((p.m + BT - 1) / BT),
                     static_cast<unsigned>((p.n + TN - 1) / TN));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (p.flags & GLQ_FLAG_NO_PDL) ? 1 : 2;
  return cudaLaunchKernelEx(&cfg, tc_linear_kernel<T, BT, TN, STAGES, WMN, GATHER, LDG>, tmap_w, tmap_a, args);
}

// K-major W rows that TMA cannot address: the LDG kernels (128-row tiles).
template <typename T>
cudaError_t launch_ldg(const Problem& p, int split, int tile_t, int tile_n, int stages, unsigned int* err,
                       cudaStream_t s) {
  if (tile_n != 128) return cudaErrorInvalidValue;
  if (stages == kPairStages) {
    switch (tile_t) {
      case 16: return launch_typed<T, 16, 128, kPairStages, false, false, true>(p, split, nullptr, err, s);
      case 32: return launch_typed<T, 32, 128, kPairStages, false, false, true>(p, split, nullptr, err, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (tile_t) {
    case 16: return launch_typed<T, 16, 128, 8, false, false, true>(p, split, nullptr, err, s);
    case 32: return launch_typed<T, 32, 128, 8, false, false, true>(p, split, nullptr, err, s);
    case 64: return launch_typed<T, 64, 128, 8, false, false, true>(p, split, nullptr, err, s);
    case 128: return launch_typed<T, 128, 128, 6, false, false, true>(p, split, nullptr, err, s);
    case 256: return launch_typed<T, 256, 128, 4, false, false, true>(p, split, nullptr, err, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, bool WMN, bool GATHER>
cudaError_t launch_bt(const Problem& p, int split, int tile_t, int tile_n, int stages, const Gather* g,
                      unsigned int* err, cudaStream_t s) {
  if (tile_n == 256) {
    switch (tile_t) {
      case 16: return launch_typed<T, 16, 256, 4, WMN, GATHER>(p, split, g, err, s);
      case 32: return launch_typed<T, 32, 256, 4, WMN, GATHER>(p, split, g, err, s);
      case 256: return launch_typed<T, 256, 256, 3, WMN, GATHER>(p, split, g, err, s);
      default: return cudaErrorInvalidValue;
    }
  }
  if (stages == kPairStages) {
    switch (tile_t) {
      case 16: return launch_typed<T, 16, 128, kPairStages, WMN, GATHER>(p, split, g, err, s);
      case 32: return launch_typed<T, 32, 128, kPairStages, WMN, GATHER>(p, split, g, err, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (tile_t) {
    case 16: return launch_typed<T, 16, 128, 8, WMN, GATHER>(p, split, g, err, s);
    case 32: return launch_typed<T, 32, 128, 8, WMN, GATHER>(p, split, g, err, s);
    case 64: return launch_typed<T, 64, 128, 8, WMN, GATHER>(p, split, g, err, s);
    case 128: return launch_typed<T, 128, 128, 6, WMN, GATHER>(p, split, g, err, s);
    case 256: return launch_typed<T, 256, 128, 4, WMN, GATHER>(p, split, g, err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t tc_prepare_device() {
  cudaError_t e = set_attrs_all<__half>();
  if (e != cudaSuccess) return e;
  return set_attrs_all<__nv_bfloat16>();
}

cudaError_t launch_tc(const Problem& p, int split, int tile_t, int tile_n, int stages, int w_mn,
                      const Gather* g, unsigned int* err, cudaStream_t s) {
  if (p.w_ldg) {
    if (g != nullptr || w_mn) return cudaErrorInvalidValue;
    return p.dtype == GLQ_DTYPE_BF16 ? launch_ldg<__nv_bfloat16>(p, split, tile_t, tile_n, stages, err, s)
                                     : launch_ldg<__half>(p, split, tile_t, tile_n, stages, err, s);
  }
  if (g != nullptr) {
    if (p.dtype == GLQ_DTYPE_BF16) {
      return w_mn ? launch_bt<__nv_bfloat16, true, true>(p, split, tile_t, tile_n, stages, g, err, s)
                  : launch_bt<__nv_bfloat16, false, true>(p, split, tile_t, tile_n, stages, g, err, s);
    }
    return w_mn ? launch_bt<__half, true, true>(p, split, tile_t, tile_n, stages, g, err, s)
                : launch_bt<__half, false, true>(p, split, tile_t, tile_n, stages, g, err, s);
  }
  if (p.dtype == GLQ_DTYPE_BF16) {
    return w_mn ? launch_bt<__nv_bfloat16, true, false>(p, split, tile_t, tile_n, stages, g, err, s)
                : launch_bt<__nv_bfloat16, false, false>(p, split, tile_t, tile_n, stages, g, err, s);
  }
  return w_mn ? launch_bt<__half, true, false>(p, split, tile_t, tile_n, stages, g, err, s)
              : launch_bt<__half, false, false>(p, split, tile_t, tile_n, stages, g, err, s);
}

}  // namespace glq
