// glq_tc.cu -- tcgen05 linear kernel for sm_100a (M >= 2 tokens).
//
// Computes Y[m, n] = epilogue(sum_k A[m, k] * W[n, k]) for a K-contiguous
// weight W[N, K] (the lab's B = W^T view) and K-contiguous activations
// A[M, K], FP32 accumulation in tensor memory, one FP16/BF16 store.
//
// Design (swap-AB, decode shapes are weight-bandwidth bound):
//   * W rows fill the 128-lane MMA M dimension; the token batch is the MMA N
//     dimension (16..256), so M = 1..128 tokens cost one W pass.
//   * One CTA = 128 threads owns a 128-row W tile x a token tile x one
//     contiguous range of 64-wide K blocks.  Warp 0 lane 0 issues TMA loads
//     (128-byte swizzle, K-major) into a STAGES-deep mbarrier ring; warp 1
//     allocates TMEM and lane 0 issues tcgen05.mma; all four warps run the
//     epilogue from TMEM (lane = W row, column = token).
//   * Split-K: the K ranges of one tile are the CTAs of one thread-block
//     cluster.  After the main loop each CTA stages its FP32 partial tile in
//     its own shared memory; after a cluster barrier CTA r reduces token
//     columns [r*T/S, (r+1)*T/S) by reading the S partials over DSMEM in
//     split order 0..S-1, applies bias + SiLU and stores.  The merge order is
//     fixed, so results are bitwise reproducible, and nothing waits on a flag.
//   * Every mbarrier wait is bounded (glq_ptx.cuh); on expiry the CTA raises
//     a bit in the device error word, stops issuing work, drains its own
//     in-flight TMA loads (bounded), still takes part in both cluster
//     barriers, frees TMEM and returns.
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
  return v / (1.0f + __expf(-v));  // SiLU = v * sigmoid(v)
}

constexpr int kTileN = 128;  // W rows per CTA (MMA M, TMEM lanes)
constexpr int kTileK = 64;   // K elements per stage: one 128-byte swizzle row
constexpr int kThreads = 128;
constexpr uint32_t kWTileBytes = kTileN * kTileK * 2;

template <int BT>
struct TcConfig {
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N for M=128 is 16..256 step 16");
  static constexpr uint32_t kATileBytes = BT * kTileK * 2;
  static constexpr uint32_t kStageBytes = kWTileBytes + kATileBytes;
  static constexpr int kStages = BT <= 64 ? 8 : (BT <= 128 ? 6 : 4);
  static constexpr uint32_t kTmemCols = BT < 32 ? 32 : BT;
  static constexpr uint32_t kPipeBytes = kStages * kStageBytes;
  static constexpr uint32_t kXchgBytes = BT * kTileN * 4;
  static constexpr uint32_t kBodyBytes = kPipeBytes > kXchgBytes ? kPipeBytes : kXchgBytes;
  static constexpr uint32_t kBarrierBytes = (2 * kStages + 1) * 8 + 16;
  static constexpr uint32_t kSmemBytes = 1024 + kBodyBytes + kBarrierBytes;
  static_assert(kStageBytes % 1024 == 0, "stage bases must stay 1024-B aligned");
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
};

struct TcArgs {
  int m, n, k;
  int num_kb;
  int split;
  int epilogue;
  const void* bias;
  void* y;
  long long ldy;
  float* partial;
  unsigned int* err;
};

template <typename T, int BT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_a, const TcArgs args) {
  using Cfg = TcConfig<BT>;
  constexpr int kStages = Cfg::kStages;

  extern __shared__ uint8_t smem_dyn[];
  const uint32_t raw_base = ptx::smem_addr(smem_dyn);
  const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
  uint8_t* smem = smem_dyn + pad;
  const uint32_t sbase = raw_base + pad;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBodyBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued_slot = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = args.split;
  const int s = blockIdx.x;  // split index == CTA rank in the (split,1,1) cluster
  const int tile_n = blockIdx.y;
  const int tile_t = blockIdx.z;
  const int kb_begin = static_cast<int>((static_cast<long long>(s) * args.num_kb) / split);
  const int kb_end = static_cast<int>((static_cast<long long>(s + 1) * args.num_kb) / split);
  const int nkb = kb_end - kb_begin;

  auto full_bar = [&](int i) { return ptx::smem_addr(&bars[i]); };
  auto empty_bar = [&](int i) { return ptx::smem_addr(&bars[kStages + i]); };
  const uint32_t done_bar = ptx::smem_addr(&bars[2 * kStages]);
  auto raise = [&](unsigned int bit) {
    atomicOr(args.err, bit);
    *abort_flag = 1;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      ptx::mbar_init(empty_bar(i), 1);
    }
    ptx::mbar_init(done_bar, 1);
    *abort_flag = 0;
    *issued_slot = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tmap_w);
    ptx::prefetch_tensormap(&tmap_a);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: W streamed once (evict-first), A reused (evict-last).
      const uint64_t pol_w = ptx::policy_evict_first();
      const uint64_t pol_a = ptx::policy_evict_last();
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int stage = i % kStages;
        const uint32_t round = static_cast<uint32_t>(i / kStages);
        if (round > 0 &&
            !ptx::mbar_wait_bounded(empty_bar(stage), (round - 1u) & 1u, abort_flag, kWaitBudgetNs)) {
          raise(kErrTimeoutProducer);
          break;
        }
        const uint32_t w_dst = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
        const uint32_t a_dst = w_dst + kWTileBytes;
        ptx::mbar_arrive_expect_tx(full_bar(stage), Cfg::kStageBytes);
        const int kx = (kb_begin + i) * kTileK;
        ptx::tma_load_2d(w_dst, &tmap_w, kx, tile_n * kTileN, full_bar(stage), pol_w);
        ptx::tma_load_2d(a_dst, &tmap_a, kx, tile_t * BT, full_bar(stage), pol_a);
        issued = i + 1;
      }
      *issued_slot = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: D[128 x BT] += W_tile[128 x 64] * A_tile[BT x 64]^T.
      constexpr uint32_t idesc = ptx::umma_idesc_f16(kTileN, BT, Elem<T>::kFormat);
      for (int i = 0; i < nkb; ++i) {
        const int stage = i % kStages;
        const uint32_t round = static_cast<uint32_t>(i / kStages);
        if (!ptx::mbar_wait_bounded(full_bar(stage), round & 1u, abort_flag, kWaitBudgetNs)) {
          raise(kErrTimeoutMma);
          break;
        }
        ptx::tc_fence_after_sync();
        const uint32_t w_src = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
        const uint64_t w_desc = ptx::umma_desc_k_sw128(w_src);
        const uint64_t a_desc = ptx::umma_desc_k_sw128(w_src + kWTileBytes);
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk) {
          // Each MMA consumes K = 16 (32 bytes); the descriptor start address
          // is in 16-byte units, so step by 2 inside the swizzled row.
          ptx::tc_mma_f16(tmem_d, w_desc + 2u * kk, a_desc + 2u * kk, idesc,
                          (i > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::tc_commit(empty_bar(stage));
      }
      ptx::tc_commit(done_bar);
    }
  }
  __syncwarp();

  // ---- Epilogue: all 128 threads; thread t owns TMEM lane t = W row t.
  if (!ptx::mbar_wait_bounded(done_bar, 0u, abort_flag, kWaitBudgetNs)) {
    raise(kErrTimeoutEpilogue);
  }
  __syncthreads();
  const bool aborted = *abort_flag != 0;
  ptx::tc_fence_after_sync();

  const int n_local = warp * 32 + lane;
  const long long n = static_cast<long long>(tile_n) * kTileN + n_local;
  const long long m0 = static_cast<long long>(tile_t) * BT;
  const int mr = static_cast<int>(min(static_cast<long long>(BT), args.m - m0));
  const bool n_ok = n < args.n;
  float bias_v = 0.0f;
  if (args.epilogue != GLQ_EPILOGUE_NONE && n_ok) {
    bias_v = Elem<T>::to_f(static_cast<const T*>(args.bias)[n]);
  }
  T* y = static_cast<T*>(args.y);
  const uint32_t t_row = tmem_d + (static_cast<uint32_t>(warp * 32) << 16);

  if (split == 1) {
    if (!aborted) {
      for (int c0 = 0; c0 < mr; c0 += 16) {
        uint32_t r[16];
        ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(c0), r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int mm = c0 + j;
          if (mm < mr && n_ok) {
            y[(m0 + mm) * args.ldy + n] =
                Elem<T>::from_f(apply_epilogue(__uint_as_float(r[j]), bias_v, args.epilogue));
          }
        }
      }
    }
  } else {
    // Partial tile staged as xchg[token][row] (FP32) over the drained pipeline.
    float* xchg = reinterpret_cast<float*>(smem);
    if (!aborted) {
      for (int c0 = 0; c0 < mr; c0 += 16) {
        uint32_t r[16];
        ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(c0), r);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int mm = c0 + j;
          if (mm < mr) {
            const float v = __uint_as_float(r[j]);
            xchg[mm * kTileN + n_local] = v;
            if (args.partial != nullptr && n_ok) {
              args.partial[(static_cast<long long>(s) * args.m + m0 + mm) * args.n + n] = v;
            }
          }
        }
      }
    }
    ptx::cluster_sync();
    if (!aborted) {
      const int m_lo = (s * mr) / split;
      const int m_hi = ((s + 1) * mr) / split;
      for (int mm = m_lo; mm < m_hi; ++mm) {
        const uint32_t local = ptx::smem_addr(&xchg[mm * kTileN + n_local]);
        float acc = 0.0f;
        for (int r = 0; r < split; ++r) {
          acc += ptx::ld_dsmem_f32(ptx::map_to_rank(local, static_cast<uint32_t>(r)));
        }
        if (n_ok) {
          y[(m0 + mm) * args.ldy + n] = Elem<T>::from_f(apply_epilogue(acc, bias_v, args.epilogue));
        }
      }
    }
    ptx::cluster_sync();  // peers have finished reading this CTA's partials
  }

  // ---- Teardown: after an abort, let this CTA's own TMA loads land first.
  if (aborted && warp == 0 && lane == 0) {
    const int issued = *issued_slot;
    for (int i = max(0, issued - kStages); i < issued; ++i) {
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

// 2-D K-major map: rows x cols(K) with a row pitch in bytes, box rows x 64.
bool encode_kmajor(CUtensorMap* map, CUtensorMapDataType type, const void* base, int64_t cols,
                   int64_t rows, int64_t row_pitch_bytes, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_pitch_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int BT>
cudaError_t set_attrs() {
  return cudaFuncSetAttribute(tc_linear_kernel<T, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              TcConfig<BT>::kSmemBytes);
}

template <typename T>
cudaError_t set_attrs_all() {
  cudaError_t e;
  if ((e = set_attrs<T, 16>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 32>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 64>()) != cudaSuccess) return e;
  if ((e = set_attrs<T, 128>()) != cudaSuccess) return e;
  return set_attrs<T, 256>();
}

template <typename T, int BT>
cudaError_t launch_typed(const Problem& p, int split, unsigned int* err, cudaStream_t stream) {
  constexpr int64_t esz = 2;
  CUtensorMap tmap_w, tmap_a;
  // W = B^T: rows n (pitch b_ns), K contiguous.  A: rows m (pitch a_rs).
  const int64_t w_pitch = p.n > 1 ? p.b_ns * esz : ((p.k * esz + 15) / 16) * 16;
  const int64_t a_pitch = p.m > 1 ? p.a_rs * esz : ((p.k * esz + 15) / 16) * 16;
  if (!encode_kmajor(&tmap_w, Elem<T>::kTmaType, p.b, p.k, p.n, w_pitch, kTileN) ||
      !encode_kmajor(&tmap_a, Elem<T>::kTmaType, p.a, p.k, p.m, a_pitch, BT)) {
    return cudaErrorInvalidValue;
  }
  TcArgs args;
  args.m = static_cast<int>(p.m);
  args.n = static_cast<int>(p.n);
  args.k = static_cast<int>(p.k);
  args.num_kb = static_cast<int>(tc_k_blocks(p.k));
  args.split = split;
  args.epilogue = p.epilogue;
  args.bias = p.bias;
  args.y = p.y;
  args.ldy = p.ldy;
  args.partial = p.partial;
  args.err = err;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(split), static_cast<unsigned>((p.n + kTileN - 1) / kTileN),
                     static_cast<unsigned>((p.m + BT - 1) / BT));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = TcConfig<BT>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tc_linear_kernel<T, BT>, tmap_w, tmap_a, args);
}

template <typename T>
cudaError_t launch_bt(const Problem& p, int split, int tile_t, unsigned int* err, cudaStream_t s) {
  switch (tile_t) {
    case 16: return launch_typed<T, 16>(p, split, err, s);
    case 32: return launch_typed<T, 32>(p, split, err, s);
    case 64: return launch_typed<T, 64>(p, split, err, s);
    case 128: return launch_typed<T, 128>(p, split, err, s);
    case 256: return launch_typed<T, 256>(p, split, err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t tc_prepare_device() {
  cudaError_t e = set_attrs_all<__half>();
  if (e != cudaSuccess) return e;
  return set_attrs_all<__nv_bfloat16>();
}

cudaError_t launch_tc(const Problem& p, int split, int tile_t, unsigned int* err, cudaStream_t s) {
  if (p.dtype == GLQ_DTYPE_BF16) return launch_bt<__nv_bfloat16>(p, split, tile_t, err, s);
  return launch_bt<__half>(p, split, tile_t, err, s);
}

}  // namespace glq
