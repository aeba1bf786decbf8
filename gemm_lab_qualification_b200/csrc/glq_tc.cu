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

// Operands TMA cannot address directly (RAW kernels, bits kRawW / kRawA).
// A raw row box: the stage's 64 K elements plus up to 7 elements of
// in-granule offset, i.e. nine 16-byte granules.
constexpr int kRawSpan = kTileK + 8;
constexpr uint32_t kRawRowBytes = kRawSpan * 2;  // 144
// TMA writes shared memory at 128-byte aligned addresses: the box of row
// class c (rows_per_class raw rows) starts at c slots of
// rows_per_class * 144 bytes rounded up to 128.
__host__ __device__ constexpr uint32_t raw_class_offset(int c, int rows_per_class) {
  return static_cast<uint32_t>(c) * ((static_cast<uint32_t>(rows_per_class) * kRawRowBytes + 127u) & ~127u);
}
// Raw bytes of `rows` tile rows in C classes, padding included, for the
// worst class count (only classes of fewer than 8 rows need padding).
__host__ __device__ constexpr uint32_t raw_area_bytes(int rows) {
  uint32_t most = 0;
  for (int c = 1; c <= 8; c *= 2) {
    const uint32_t b = raw_class_offset(c, rows / c);
    most = b > most ? b : most;
  }
  return most;
}
// Warps 2..5 turn raw stages into aligned ones (idle during the main loop
// otherwise): one per SM sub-partition, which is what bounds the shift.
// When both operands are raw and the token tile is small (at most 32
// tokens), warps 2..5 align W (into tensor memory) while warps 6 and 7
// align A (into shared memory), so the two shifts of a stage run side by
// side (32 x 4096 x 4090: 14.3 -> 14.0 us); a larger A tile is aligned by
// warps 2..5 before W (two warps made M = 128 slower: 24.4 -> 29.7 us).
constexpr int kShiftWarps = 4;
__host__ __device__ constexpr bool split_shift(int raw, int bt) { return raw == (kRawW | kRawA) && bt <= 32; }
__host__ __device__ constexpr int shift_warps(int raw, int bt) {
  return split_shift(raw, bt) ? kShiftWarps + 2 : raw != 0 ? kShiftWarps : 0;
}

// BT: token tile (MMA N).  TN: W rows per CTA, one M = 128 MMA (and one TMEM
// accumulator of BT columns) per 128 rows.  A 256-row tile moves W in 32 KB
// TMA boxes, which streams HBM measurably better than 16 KB boxes at equal
// bytes in flight.  STAGES: depth of the TMA ring; 4 stages of a small token
// tile plus the split-K receive buffer keep a CTA under 113 KB of shared
// memory, so two CTAs share an SM.
//
// KPS: K blocks per load stage.  With KPS = 2 (K-major, 128-row tiles, no
// raw operand) one 3-D TMA box fetches a 32 KB W stage (two 16 KB K-major
// tiles back to back) and another the two A tiles, so the W stream moves in
// 32 KB operations without doubling the tile (and the split-K merge).
//
// Shared memory: STAGES load stages (what TMA writes: for each operand its
// 128-byte-swizzled tile(s), or for a RAW operand its raw row boxes of 144
// bytes per row), then, in RAW kernels, two aligned stages holding the
// swizzled tiles of the RAW operands.
template <int BT, int TN, int STAGES, int RAW = 0, int KPS = 1>
struct TcConfig {
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N for M=128 is 16..256 step 16");
  static_assert(TN == 128 || TN == 256, "tile rows are one or two M=128 MMAs");
  static_assert(RAW == 0 || TN == 128, "raw-staged kernels use 128-row W tiles");
  static_assert(KPS == 1 || (KPS == 2 && RAW == 0 && TN == 128), "two K blocks per stage: plain 128-row tiles");
  static constexpr bool kRawW_ = (RAW & kRawW) != 0;
  static constexpr bool kRawA_ = (RAW & kRawA) != 0;
  static constexpr int kAcc = TN / 128;
  static constexpr int kKps = KPS;
  static constexpr uint32_t kWTileBytes = TN * kTileK * 2;  // one K block
  static constexpr uint32_t kATileBytes = BT * kTileK * 2;  // one K block
  // Load stage: the W part first, then A (1024-byte aligned when swizzled).
  static constexpr uint32_t kLoadWBytes = kRawW_ ? raw_area_bytes(TN) : KPS * kWTileBytes;
  static constexpr uint32_t kLoadABytes = kRawA_ ? raw_area_bytes(BT) : KPS * kATileBytes;
  // Bytes TMA lands per stage (every box counts in full, zero fill included).
  static constexpr uint32_t kLoadTx =
      (kRawW_ ? TN * kRawRowBytes : KPS * kWTileBytes) + (kRawA_ ? BT * kRawRowBytes : KPS * kATileBytes);
  // Load stages holding a swizzled tile start 1024-byte aligned; raw-only
  // stages need the TMA's 128 bytes.
  static constexpr uint32_t kStageAlign = (kRawW_ && kRawA_) ? 128u : 1024u;
  static constexpr uint32_t kStageBytes = (kLoadWBytes + kLoadABytes + kStageAlign - 1u) / kStageAlign * kStageAlign;
  static constexpr int kStages = STAGES;
  // Aligned stages of the RAW kernels: two, so that the shift of stage i + 1
  // overlaps the MMA of stage i.  A raw W tile is aligned into tensor
  // memory (the MMA's A operand: TMEM lane = tile row, 32 columns of two
  // 16-bit elements per stage, past the accumulators); a raw A tile into
  // a swizzled shared-memory stage.
  static constexpr int kShift = RAW == 0 ? 0 : 2;
  static constexpr uint32_t kShiftBytes = kRawA_ ? kATileBytes : 0u;
  static constexpr uint32_t kShiftBase = (kStages * kStageBytes + 1023u) / 1024u * 1024u;
  static constexpr uint32_t kAccCols = kAcc * BT;
  static constexpr uint32_t kWTmemCol = (kAccCols + 31u) / 32u * 32u;  // first column of the W stages
  static constexpr uint32_t kWTmemStageCols = kTileK / 2;               // 64 elements per row
  static constexpr uint32_t kUsedCols = kRawW_ ? kWTmemCol + kShift * kWTmemStageCols : kAccCols;
  static constexpr uint32_t kTmemCols =
      kUsedCols <= 32 ? 32 : (kUsedCols <= 64 ? 64 : (kUsedCols <= 128 ? 128 : (kUsedCols <= 256 ? 256 : 512)));
  static_assert(kUsedCols <= 512, "tensor memory holds 512 columns");
  static constexpr uint32_t kPipeBytes = kShiftBase + kShift * kShiftBytes;
  // full/empty per load stage, full/empty per aligned stage, done, receive.
  static constexpr int kBars = 2 * kStages + 2 * kShift + 2;
  static constexpr uint32_t kBarrierBytes = kBars * 8 + 16;
  static_assert(kLoadWBytes % 1024 == 0, "the A part of a load stage must stay 1024-B aligned");
  static_assert(kShiftBytes % 1024 == 0, "aligned stages must stay 1024-B aligned");
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
  int w_3d;                 // MN-major W (WMN): one 3-D box per stage instead of TN / 64 2-D boxes
  // RAW kernels: rows of a raw operand are split into C classes (row
  // r in class r % C, C a power of two); class c's rows start s_c elements
  // into a 16-byte granule, 4 bits per class in *_shifts.
  int w_classes, a_classes;
  unsigned int w_shifts, a_shifts;
};

// Tensor maps of a launch.  Plain kernels use w[0] and a[0]; a RAW operand
// has one map per row class (unused classes repeat class 0).
template <int RAW>
struct alignas(64) TmaSet {
  CUtensorMap w[(RAW & kRawW) ? kMaxClasses : 1];
  CUtensorMap a[(RAW & kRawA) ? kMaxClasses : 1];
};

// ---- Raw-staged operands (RAW kernels).
//
// A K-contiguous operand whose base or row pitch P (elements) is not 16-byte
// aligned cannot be a TMA source as it is, but every class of rows
// r == c (mod C) can: with C a power of two such that C * P is a multiple of
// 8 elements, the rows of class c sit C * P elements apart (a 16-byte
// multiple), and the class's first row starts E_c = b0 + c * P elements past
// the 16-byte boundary below the operand's base (b0 = the base's offset in
// elements).  The host encodes one 2-D map per class whose origin is that
// boundary plus (E_c & ~7) elements; a row's element k then sits at
// x = k + s_c with s_c = E_c & 7, and the map's inner extent is K + s_c, so
// TMA zero-fills exactly the columns k >= K.  The rows of a tile (W: 128
// rows n0.., A: BT rows t0.., both multiples of 8) split into the C classes
// as contiguous runs of class rows, so a stage is C boxes of
// (rows / C) x 72 elements: the 64 K elements of the stage plus room for
// the shift, landed unswizzled, row i of class c at i * 144 bytes past the
// start of class c's box (raw_class_offset: every box starts 128-byte
// aligned).  (C * P >= K + 8 is required, so that a class's rows never
// overlap.)
//
// The shift warps (2..5) then write each row's 64 elements, shifted by s_c,
// into the 128-byte-swizzled K-major tile the MMA reads: 16-byte chunk g of
// a row is taken from its raw granules g and g + 1.  The chunks equal what
// a TMA load with zero fill writes from an aligned copy of the operand, so
// the MMA sums the same values in the same order.

// 16 bytes starting S elements into the 32-byte window lo:hi.
template <int S>
__device__ __forceinline__ uint4 shift_by(const uint4& lo, const uint4& hi) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  constexpr int q = S >> 1;  // whole 32-bit words
  if constexpr ((S & 1) == 0) {
    return make_uint4(w[q], w[q + 1], w[q + 2], w[q + 3]);
  } else {  // plus one element
    return make_uint4(__funnelshift_r(w[q], w[q + 1], 16), __funnelshift_r(w[q + 1], w[q + 2], 16),
                      __funnelshift_r(w[q + 2], w[q + 3], 16), __funnelshift_r(w[q + 3], w[q + 4], 16));
  }
}

// The same for a per-lane shift, without branches: words s / 2 .. s / 2 + 4
// of the window picked by two levels of selects, then each output word is
// the byte permutation of two neighbours (a half-word shift for odd s).
__device__ __forceinline__ uint4 shift_window(const uint4& lo, const uint4& hi, unsigned s) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  const bool q1 = (s & 2u) != 0, q2 = (s & 4u) != 0;
  uint32_t p[5];
#pragma unroll
  for (int e = 0; e < 5; ++e) {
    const uint32_t low = q1 ? w[e + 1] : w[e];
    const uint32_t high = q1 ? w[e + 3] : w[e + 2];
    p[e] = q2 ? high : low;  // w[e + s / 2]
  }
  const unsigned sel = (s & 1u) ? 0x5432u : 0x3210u;
  return make_uint4(__byte_perm(p[0], p[1], sel), __byte_perm(p[1], p[2], sel), __byte_perm(p[2], p[3], sel),
                    __byte_perm(p[3], p[4], sel));
}

// A batch of N chunks that share the shift S: shift and store.
template <int S, int N>
__device__ __forceinline__ void store_shifted(const uint4 (&lo)[N], const uint4 (&hi)[N], uint8_t* const (&out)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) *reinterpret_cast<uint4*>(out[j]) = shift_by<S>(lo[j], hi[j]);
}

// Rows [0, ROWS) of one raw load stage -> the swizzled K-major tile at dst,
// by the NW shift warps W0, W0 + 1, ...  Raw rows are taken in class order
// in warp steps of four rows (lane l: row l / 8 of the four, chunk
// g = l % 8); shift warp w takes the contiguous block of steps
// [w * ROWS / (4 NW), (w + 1) * ROWS / (4 NW)), in batches of up to four
// steps.  A batch of 16 rows inside one class (every
// W batch) has a warp-uniform shift, applied by a compile-time shift chosen
// once per batch; batches that span classes (A tiles of 16 or 32 tokens in
// 4 or 8 classes) shift per lane.  Each lane loads its two raw granules
// itself.  `release` runs once every raw granule of this operand is in
// registers, before the last batch is shifted and stored, so the load stage
// is freed early.
template <int ROWS, int NW = kShiftWarps, int W0 = 2, int MAXB = 4, typename Release>
__device__ __forceinline__ void shift_rows(const uint8_t* raw, uint8_t* dst, int classes, unsigned shifts,
                                           Release release) {
  static_assert(ROWS % (4 * NW) == 0, "tile rows come in multiples of four per shift warp");
  constexpr int kPerWarp = ROWS / (4 * NW);                  // warp steps per shift warp
  constexpr int kBatch = kPerWarp < MAXB ? kPerWarp : MAXB;  // steps whose loads are issued together
  static_assert(kPerWarp % kBatch == 0, "batches stay inside one shift warp's block of steps");
  const int wq = (static_cast<int>(threadIdx.x) >> 5) - W0;  // shift warp 0..NW-1
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  const int log_c = classes == 1 ? 0 : classes == 2 ? 1 : classes == 4 ? 2 : 3;
  constexpr int kLogRows = ROWS == 16 ? 4 : ROWS == 32 ? 5 : ROWS == 64 ? 6 : ROWS == 128 ? 7 : 8;
  static_assert((1 << kLogRows) == ROWS, "tile rows are a power of two");
  const int log_rpc = kLogRows - log_c;  // rows per class = ROWS / C
  const bool uniform = (1 << log_rpc) >= 4 * kBatch;  // a batch's rows lie in one class
#pragma unroll
  for (int b = 0; b < kPerWarp; b += kBatch) {
    uint4 lo[kBatch], hi[kBatch];
    uint8_t* out[kBatch];
    unsigned sh[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int idx = 4 * (wq * kPerWarp + b + j) + (lane >> 3);  // class-order row index
      const int c = idx >> log_rpc;
      const int i = idx - (c << log_rpc);
      const int rho = (i << log_c) + c;  // tile row
      sh[j] = (shifts >> (4 * c)) & 7u;
      out[j] = dst + rho * 128 + ((g ^ (rho & 7)) << 4);
      const uint8_t* row = raw + raw_class_offset(c, 1 << log_rpc) + i * kRawRowBytes + 16 * g;
      lo[j] = *reinterpret_cast<const uint4*>(row);
      hi[j] = *reinterpret_cast<const uint4*>(row + 16);
    }
    if (b + kBatch >= kPerWarp) release();
    if (uniform) {
      switch (sh[0]) {
        case 0: store_shifted<0>(lo, hi, out); break;
        case 1: store_shifted<1>(lo, hi, out); break;
        case 2: store_shifted<2>(lo, hi, out); break;
        case 3: store_shifted<3>(lo, hi, out); break;
        case 4: store_shifted<4>(lo, hi, out); break;
        case 5: store_shifted<5>(lo, hi, out); break;
        case 6: store_shifted<6>(lo, hi, out); break;
        default: store_shifted<7>(lo, hi, out); break;
      }
    } else {
#pragma unroll
      for (int j = 0; j < kBatch; ++j) *reinterpret_cast<uint4*>(out[j]) = shift_window(lo[j], hi[j], sh[j]);
    }
  }
}

// Eight 16-byte chunks of one raw row (granules g and g + 1 for chunk g),
// shifted by S elements, as the 32 TMEM columns of that row.
template <int S>
__device__ __forceinline__ void shift_row(const uint4 (&gr)[9], uint32_t (&lo)[16], uint32_t (&hi)[16]) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const uint4 v = shift_by<S>(gr[g], gr[g + 1]);
    uint32_t* out = g < 4 ? lo + 4 * g : hi + 4 * (g - 4);
    out[0] = v.x;
    out[1] = v.y;
    out[2] = v.z;
    out[3] = v.w;
  }
}

// A raw W load stage (TN = 128 rows) -> one aligned W stage in tensor
// memory.  Lane l of the shift warp on TMEM sub-partition q = warp % 4
// converts TMEM lane lam = 32 q + l, which holds row i of class c in
// class-major order (lam = c * R + i, R = 128 / C rows per class), i.e.
// tile row i * C + c: it loads that row's nine raw granules (consecutive
// lanes read rows 144 B apart, free of bank conflicts), releases the load
// stage once every lane has them, shifts them by the class's s_c and
// writes the 64 elements as 32 TMEM columns of its lane.  With C <= 4 a
// warp's 32 lanes share one class (a compile-time shift chosen once per
// warp); with C = 8 the two half-warps shift by their own class's s_c.
template <typename Release>
__device__ __forceinline__ void shift_w_tmem(const uint8_t* raw, uint32_t tmem_stage, int classes, unsigned shifts,
                                             Release release) {
  const int q = (static_cast<int>(threadIdx.x) >> 5) & 3;
  const int lane = threadIdx.x & 31;
  const int lam = 32 * q + lane;
  const int log_c = classes == 1 ? 0 : classes == 2 ? 1 : classes == 4 ? 2 : 3;
  const int log_r = 7 - log_c;
  const int c = lam >> log_r;
  const int i = lam & ((1 << log_r) - 1);
  const uint8_t* row = raw + raw_class_offset(c, 1 << log_r) + i * kRawRowBytes;
  uint4 gr[9];
#pragma unroll
  for (int g = 0; g < 9; ++g) gr[g] = *reinterpret_cast<const uint4*>(row + 16 * g);
  release();
  const unsigned sh = (shifts >> (4 * c)) & 7u;
  uint32_t lo[16], hi[16];
  switch (sh) {
    case 0: shift_row<0>(gr, lo, hi); break;
    case 1: shift_row<1>(gr, lo, hi); break;
    case 2: shift_row<2>(gr, lo, hi); break;
    case 3: shift_row<3>(gr, lo, hi); break;
    case 4: shift_row<4>(gr, lo, hi); break;
    case 5: shift_row<5>(gr, lo, hi); break;
    case 6: shift_row<6>(gr, lo, hi); break;
    default: shift_row<7>(gr, lo, hi); break;
  }
  // The collective stores need the whole warp (the half-warps of C = 8 may
  // have taken different cases above).
  __syncwarp();
  const uint32_t taddr = tmem_stage + (static_cast<uint32_t>(32 * q) << 16);
  ptx::tmem_st_32x32b_x16(taddr, lo);
  ptx::tmem_st_32x32b_x16(taddr + 16u, hi);
}

// Tile row of TMEM lane `lam` in a raw W tile (class-major lane order, see
// shift_w_tmem).
__device__ __forceinline__ int raw_w_tile_row(int lam, int classes) {
  const int log_c = classes == 1 ? 0 : classes == 2 ? 1 : classes == 4 ? 2 : 3;
  const int log_r = 7 - log_c;
  return ((lam & ((1 << log_r) - 1)) << log_c) + (lam >> log_r);
}

// The shift warps' loop: for every K block of this CTA, wait for its load
// stage and a free aligned stage, write the RAW operands' aligned tiles (A
// swizzled in shared memory, W in tensor memory), release the load stage
// (one arrival per warp: the raw bytes are read) and publish the aligned
// stage (every thread's writes made visible to the tensor core by its own
// proxy fence or TMEM store wait, then one arrival per warp).
template <int BT, int TN, int STAGES, int RAW, typename FullBar, typename EmptyBar, typename SFullBar,
          typename SEmptyBar, typename Raise>
__device__ __forceinline__ void shift_loop(const TcArgs& args, uint8_t* smem, uint32_t tmem_d, int nkb,
                                           FullBar full_bar, EmptyBar empty_bar, SFullBar sfull_bar,
                                           SEmptyBar sempty_bar, const volatile int* abort_flag, Raise raise) {
  using Cfg = TcConfig<BT, TN, STAGES, RAW>;
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < nkb; ++i) {
    const int stage = i % Cfg::kStages;
    const int sst = i % Cfg::kShift;
    bool ok = true;
    if (lane == 0) {
      ok = ptx::mbar_wait_bounded(full_bar(stage), static_cast<uint32_t>(i / Cfg::kStages) & 1u, abort_flag,
                                  kWaitBudgetNs);
      if (ok && i >= Cfg::kShift) {
        ok = ptx::mbar_wait_bounded(sempty_bar(sst), static_cast<uint32_t>(i / Cfg::kShift - 1) & 1u, abort_flag,
                                    kWaitBudgetNs);
      }
    }
    if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) {
      if (lane == 0) raise(kErrTimeoutProducer);
      return;
    }
    // The MMAs that read this aligned stage have completed (their commit
    // released sempty): order this warp's TMEM stores after them.
    if constexpr (Cfg::kRawW_) ptx::tc_fence_after_sync();
    const uint8_t* load = smem + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
    uint8_t* aligned = smem + Cfg::kShiftBase + static_cast<uint32_t>(sst) * Cfg::kShiftBytes;
    // The load stage is released (one arrival per shift warp) once that
    // warp's raw granules are in registers.
    auto release = [&]() {
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(empty_bar(stage));
    };
    auto keep = []() {};
    constexpr bool kSplit = split_shift(RAW, BT);
    // With the split, warps 6..7 align A and warps 2..5 align W; otherwise
    // warps 2..5 align A (if raw), then W (if raw).
    const bool a_warp = kSplit && (threadIdx.x >> 5) >= 2 + kShiftWarps;
    if constexpr (kSplit) {
      if (a_warp) {
        // Batches of two steps (8 rows) keep a batch inside one row class
        // for A tiles of 32 tokens in 4 classes.
        shift_rows<BT, 2, 2 + kShiftWarps, 2>(load + Cfg::kLoadWBytes, aligned, args.a_classes, args.a_shifts,
                                              release);
        ptx::fence_proxy_async_smem();
      }
    } else if constexpr (Cfg::kRawA_) {
      if constexpr (Cfg::kRawW_) {
        shift_rows<BT>(load + Cfg::kLoadWBytes, aligned, args.a_classes, args.a_shifts, keep);
      } else {
        shift_rows<BT>(load + Cfg::kLoadWBytes, aligned, args.a_classes, args.a_shifts, release);
      }
      ptx::fence_proxy_async_smem();
    }
    if constexpr (Cfg::kRawW_) {
      static_assert(TN == 128, "raw W tiles are one M = 128 MMA");
      if (!a_warp) {
        shift_w_tmem(load, tmem_d + Cfg::kWTmemCol + static_cast<uint32_t>(sst) * Cfg::kWTmemStageCols,
                     args.w_classes, args.w_shifts, release);
        ptx::tmem_st_wait();
        ptx::tc_fence_before_sync();
      }
    }
    // Every writer orders its stores before the tensor core's reads (proxy
    // fence or TMEM store wait above), then one arrival per warp (128
    // arrivals on one barrier serialise).
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(sfull_bar(sst));
  }
}

// RAW: operands TMA cannot address are staged raw and aligned by warps 2..5
// (K-major W, 128-row tiles, no gather); two CTAs per SM must still fit, so
// these instantiations are capped at 128 registers.
template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, int RAW = 0, int KPS = 1>
__global__ void __launch_bounds__(kThreads, RAW != 0 ? 2 : 1)
    tc_linear_kernel(const __grid_constant__ TmaSet<RAW> maps, const TcArgs args) {
  static_assert(RAW == 0 || (!WMN && !GATHER && TN == 128), "raw-staged operands: K-major 128-row tiles only");
  using Cfg = TcConfig<BT, TN, STAGES, RAW, KPS>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kShift = Cfg::kShift;
  // The MMA reads a load stage directly unless both operands are raw.
  constexpr bool kMmaReadsLoad = !(Cfg::kRawW_ && Cfg::kRawA_);

  extern __shared__ uint8_t smem_dyn[];
  const uint32_t raw_base = ptx::smem_addr(smem_dyn);
  const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
  uint8_t* smem = smem_dyn + pad;
  const uint32_t sbase = raw_base + pad;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + args.barrier_offset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kBars);
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
  // Load stages of this CTA (KPS K blocks each; the planner gives every CTA
  // a multiple of KPS blocks).
  const int nst = (nkb + KPS - 1) / KPS;

  auto full_bar = [&](int i) { return ptx::smem_addr(&bars[i]); };
  auto empty_bar = [&](int i) { return ptx::smem_addr(&bars[kStages + i]); };
  auto sfull_bar = [&](int i) { return ptx::smem_addr(&bars[2 * kStages + i]); };
  auto sempty_bar = [&](int i) { return ptx::smem_addr(&bars[2 * kStages + kShift + i]); };
  const uint32_t done_bar = ptx::smem_addr(&bars[2 * kStages + 2 * kShift]);
  const uint32_t recv_bar = ptx::smem_addr(&bars[2 * kStages + 2 * kShift + 1]);

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
    const int k0 = (kb_begin + i * KPS) * kTileK;
    ptx::mbar_arrive_expect_tx(full_bar(stage), Cfg::kLoadTx);
    if constexpr (Cfg::kRawW_) {
      // One box of TN / C rows x 72 elements per row class, unswizzled.
      const int rows = TN / args.w_classes;
      for (int c = 0; c < args.w_classes; ++c) {
        ptx::tma_load_2d(w_dst + raw_class_offset(c, rows), &maps.w[c], k0,
                         tile_n * rows, full_bar(stage), pol_w);
      }
    } else if constexpr (WMN) {
      if (KPS == 2 || args.w_3d) {
        // One box of 64 N-contiguous W rows x 64 * KPS K rows x TN / 64
        // column blocks: the column blocks land 64 * KPS * 128 B apart.
        ptx::tma_load_3d(w_dst, &maps.w[0], 0, k0, tile_n * (TN / 64), full_bar(stage), pol_w);
      } else {
        // TN/64 boxes of 64 N-contiguous W rows x 64 K rows, 8 KB apart.
#pragma unroll
        for (int j = 0; j < TN / 64; ++j) {
          ptx::tma_load_2d(w_dst + static_cast<uint32_t>(j) * kMnBoxBytes, &maps.w[0], tile_n * TN + 64 * j, k0,
                           full_bar(stage), pol_w);
        }
      }
    } else if constexpr (KPS == 2) {
      // One 64 x TN x 2 box: two K-major tiles of consecutive K blocks.
      ptx::tma_load_3d(w_dst, &maps.w[0], 0, tile_n * TN, kb_begin + i * KPS, full_bar(stage), pol_w);
    } else {
      ptx::tma_load_2d(w_dst, &maps.w[0], k0, tile_n * TN, full_bar(stage), pol_w);
    }
  };
  auto issue_a = [&](int i) {
    const int stage = i % kStages;
    const uint32_t a_dst = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes + Cfg::kLoadWBytes;
    const int k0 = (kb_begin + i * KPS) * kTileK;
    if constexpr (Cfg::kRawA_) {
      const int rows = BT / args.a_classes;
      for (int c = 0; c < args.a_classes; ++c) {
        ptx::tma_load_2d(a_dst + raw_class_offset(c, rows), &maps.a[c], k0,
                         tile_t * rows, full_bar(stage), pol_a);
      }
    } else if constexpr (KPS == 2) {
      ptx::tma_load_3d(a_dst, &maps.a[0], 0, tile_t * BT, kb_begin + i * KPS, full_bar(stage), pol_a);
    } else {
      ptx::tma_load_2d(a_dst, &maps.a[0], k0, tile_t * BT, full_bar(stage), pol_a);
    }
  };
  auto issue = [&](int i) {
    issue_w(i);
    issue_a(i);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      // A load stage is free once the MMA has read it (tcgen05.commit) and,
      // in RAW kernels, once every shift warp has read its raw rows.
      ptx::mbar_init(empty_bar(i), shift_warps(RAW, BT) + (kMmaReadsLoad ? 1 : 0));
    }
    for (int i = 0; i < kShift; ++i) {
      ptx::mbar_init(sfull_bar(i), shift_warps(RAW, BT));
      ptx::mbar_init(sempty_bar(i), 1);
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
    for (int c = 0; c < ((RAW & kRawW) ? args.w_classes : 1); ++c) ptx::prefetch_tensormap(&maps.w[c]);
    for (int c = 0; c < ((RAW & kRawA) ? args.a_classes : 1); ++c) ptx::prefetch_tensormap(&maps.a[c]);
    pol_w = ptx::policy_evict_first();
    pol_a = ptx::policy_evict_last();
    // Start the stream before anything else: the first kStages stages are
    // free, so these loads need no wait.  With programmatic dependent launch
    // the predecessor kernel may still be running: A (and W unless the
    // caller declared the weights static) is read only after the dependency
    // wait.
    const int first = nst < kStages ? nst : kStages;
    const bool static_w = RAW == 0 && (args.flags & GLQ_FLAG_STATIC_WEIGHTS) != 0;
    if (static_w) {
      for (int i = 0; i < first; ++i) issue_w(i);
    }
    ptx::grid_dependency_wait();
    for (; issued < first; ++issued) {
      if (!static_w) issue_w(issued);
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
  const int n_local = acc_idx * 128 + lane_group * 32 + lane;  // TMEM lane == threadIdx.x % TN
  // The W row a TMEM lane holds: lane = tile row, except for a raw W tile
  // (class-major lane order).  The split-K merge pairs partials by TMEM
  // lane (every CTA of a cluster orders its rows the same way); the output
  // and the bias use the W row.
  int w_row = n_local;
  if constexpr (Cfg::kRawW_) w_row = raw_w_tile_row(n_local, args.w_classes);
  const long long n = static_cast<long long>(tile_n) * TN + w_row;
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
  // The shift warps (RAW) wait after their loop instead.
  const bool shifter = RAW != 0 && warp >= 2 && warp < 2 + shift_warps(RAW, BT);
  if (recv_dedicated) {
    ptx::cluster_arrive_relaxed();
    if (warp >= 2 && !shifter) ptx::cluster_wait();
  }

  if (warp == 0) {
    if (lane == 0) {
      for (int i = issued; i < nst; ++i) {
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
      for (int i = 0; i < nst; ++i) {
        const int stage = i % kStages;
        const uint32_t round = static_cast<uint32_t>(i / kStages);
        const int sst = kShift > 0 ? i % kShift : 0;
        bool ok = true;
        if (kMmaReadsLoad) ok = ptx::mbar_wait_bounded(full_bar(stage), round & 1u, abort_flag, kWaitBudgetNs);
        if (kShift > 0 && ok) {
          ok = ptx::mbar_wait_bounded(sfull_bar(sst), static_cast<uint32_t>(i / (kShift > 0 ? kShift : 1)) & 1u,
                                      abort_flag, kWaitBudgetNs);
        }
        if (!ok) {
          raise(kErrTimeoutMma);
          break;
        }
        ptx::tc_fence_after_sync();
        const uint32_t load = sbase + static_cast<uint32_t>(stage) * Cfg::kStageBytes;
        const uint32_t aligned = sbase + Cfg::kShiftBase + static_cast<uint32_t>(sst) * Cfg::kShiftBytes;
        const uint32_t a_src = Cfg::kRawA_ ? aligned : load + Cfg::kLoadWBytes;
        const uint64_t a_desc = ptx::umma_desc_k_sw128(a_src);
        if constexpr (Cfg::kRawW_) {
          // W from tensor memory: 8 columns (16 K elements) per MMA.
          const uint32_t w_tmem = tmem_d + Cfg::kWTmemCol + static_cast<uint32_t>(sst) * Cfg::kWTmemStageCols;
#pragma unroll
          for (int kk = 0; kk < kTileK / 16; ++kk) {
            ptx::tc_mma_f16_ts(tmem_d, w_tmem + 8u * kk, a_desc + 2u * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
        } else {
          // MN-major boxes of two K blocks put the 64-element column blocks
          // 16 KB apart and the second K block 8 KB into each.
          const uint64_t w_desc =
              WMN ? ptx::umma_desc_mn_sw128(load, KPS * kMnBoxBytes) : ptx::umma_desc_k_sw128(load);
          constexpr uint32_t kWBlockStep = WMN ? (kMnBoxBytes >> 4) : (Cfg::kWTileBytes >> 4);
#pragma unroll
          for (int j = 0; j < KPS; ++j) {
            // K block j of the stage: its W and A tiles follow those of
            // block j - 1 (descriptor addresses in 16-byte units).
            if (j > 0 && i * KPS + j >= nkb) break;
#pragma unroll
            for (int kk = 0; kk < kTileK / 16; ++kk) {
              // Each MMA consumes K = 16.  The 128-row halves of a 256-row W
              // tile are 16 KB (1024 units) apart in both layouts.
#pragma unroll
              for (int h = 0; h < Cfg::kAcc; ++h) {
                ptx::tc_mma_f16(tmem_d + static_cast<uint32_t>(h * BT),
                                w_desc + kWBlockStep * j + 1024u * KPS * h + kWStep * kk,
                                a_desc + (Cfg::kATileBytes >> 4) * j + 2u * kk, idesc,
                                (i > 0 || j > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
        }
        if (kShift > 0) ptx::tc_commit(sempty_bar(sst));
        if (kMmaReadsLoad) ptx::tc_commit(empty_bar(stage));
      }
      ptx::tc_commit(done_bar);
    }
  } else if (shifter) {
    if constexpr (RAW != 0) {
      shift_loop<BT, TN, STAGES, RAW>(args, smem, tmem_d, nkb, full_bar, empty_bar, sfull_bar, sempty_bar,
                                      abort_flag, raise);
    }
  }
  __syncwarp();
  if (recv_dedicated && (warp < 2 || shifter)) ptx::cluster_wait();

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

// 3-D map of a row-major matrix rows x k (K contiguous, k a multiple of 64)
// seen as [k / 64 blocks][rows][64]: dims {64, rows, k / 64}, strides
// {row pitch, 128 bytes}; a box of 64 x box_rows x 2 lands as two
// consecutive 128-byte-swizzled K-major tiles (two K blocks), which is what
// two 2-D boxes of 64 x box_rows at consecutive K blocks would give.
bool encode_kblocks_3d(CUtensorMap* map, CUtensorMapDataType type, const void* base, int64_t k, int64_t rows,
                       int64_t row_pitch_bytes, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encoder();
  if (encode == nullptr || k % kTileK != 0) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kTileK), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(k / kTileK)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_pitch_bytes), static_cast<cuuint64_t>(kTileK * 2)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTileK), box_rows, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, type, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map of the lab's B = [K, N] (N contiguous, n a multiple of 64) seen
// as [n / 64 column blocks][k][64]: dims {64, k, n / 64}, strides {row pitch,
// 128 bytes}; a box of 64 x box_k x box_blocks lands box_blocks MN-major
// 128-byte-swizzled tiles of 64 columns x box_k rows back to back, which is
// what box_blocks 2-D boxes of 64 x box_k would write.
bool encode_mn_3d(CUtensorMap* map, CUtensorMapDataType type, const void* base, int64_t n, int64_t k,
                  int64_t row_pitch_bytes, uint32_t box_k, uint32_t box_blocks) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encoder();
  if (encode == nullptr || n % 64 != 0) return false;
  const cuuint64_t dims[3] = {64u, static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(n / 64)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_pitch_bytes), 128u};
  const cuuint32_t box[3] = {64u, box_k, box_blocks};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, type, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// One map per row class of a raw operand (rows x k, K contiguous, row pitch
// `pitch` elements, 2-byte aligned base): class c's rows r = c, c + C, ...
// as a 2-D tensor of (k + s_c) x rows_c elements, origin at the 16-byte
// boundary at or below its first row's start, row pitch C * pitch; boxes of
// (tile_rows / C) rows x kRawSpan, unswizzled, zero fill out of bounds.  A
// class without rows repeats class 0's map: what it loads lands on tile rows
// past the operand's end, whose results are never stored.
bool encode_raw(CUtensorMap* maps, CUtensorMapDataType type, const void* base, int64_t rows, int64_t k,
                int64_t pitch, int tile_rows, RawClasses* rc) {
  if (!raw_classes(base, rows, k, pitch, rc)) return false;
  PFN_cuTensorMapEncodeTiled_v12000 encode = encoder();
  if (encode == nullptr) return false;
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  const uintptr_t b_aligned = b & ~static_cast<uintptr_t>(15);
  const int64_t b0 = static_cast<int64_t>((b & 15u) >> 1);
  const int64_t pe = raw_pitch(rows, k, pitch);
  const int c_count = rc->classes;
  for (int c = 0; c < kMaxClasses; ++c) {
    const int64_t rows_c = c < c_count ? (rows - c + c_count - 1) / c_count : 0;
    if (rows_c <= 0) {
      maps[c] = maps[0];
      continue;
    }
    const int64_t e = b0 + c * pe;
    const int64_t s = e & 7;
    void* origin = reinterpret_cast<void*>(b_aligned + static_cast<uintptr_t>((e - s) * 2));
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k + s), static_cast<cuuint64_t>(rows_c)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(c_count * pe * 2)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRawSpan), static_cast<cuuint32_t>(tile_rows / c_count)};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&maps[c], type, 2, origin, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return false;
    }
  }
  return true;
}

// Load-ring depth of the RAW kernels at two CTAs per SM: with one raw
// operand the plain kernel's four stages fit (a raw W tile is aligned into
// tensor memory, so it takes no aligned shared-memory stage); with both, a
// stage holds both raw areas and three fit beside the two aligned A stages
// and the split-K receive buffer.
constexpr int raw_pair_stages(int raw) { return raw == (kRawW | kRawA) ? 3 : kPairStages; }

template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, int RAW = 0, int KPS = 1>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(tc_linear_kernel<T, BT, TN, STAGES, WMN, GATHER, RAW, KPS>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
}

template <typename T, bool WMN>
cudaError_t set_attrs_kps2() {
  cudaError_t e;
  if ((e = set_attr<T, 16, 128, kPairStagesKps2, WMN, false, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 32, 128, kPairStagesKps2, WMN, false, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 16, 128, kPairStagesKps2, WMN, true, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 32, 128, kPairStagesKps2, WMN, true, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 64, 128, 4, WMN, false, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 64, 128, 4, WMN, true, 0, 2>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 128, 128, 3, WMN, false, 0, 2>()) != cudaSuccess) return e;
  return set_attr<T, 128, 128, 3, WMN, true, 0, 2>();
}

template <typename T, int RAW>
cudaError_t set_attrs_raw() {
  cudaError_t e;
  constexpr int kPair = raw_pair_stages(RAW);
  if ((e = set_attr<T, 16, 128, kPair, false, false, RAW>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 32, 128, kPair, false, false, RAW>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 16, 128, 8, false, false, RAW>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 32, 128, 8, false, false, RAW>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 64, 128, 6, false, false, RAW>()) != cudaSuccess) return e;
  if ((e = set_attr<T, 128, 128, 4, false, false, RAW>()) != cudaSuccess) return e;
  return set_attr<T, 256, 128, 2, false, false, RAW>();
}

template <typename T, int BT, int TN, int STAGES>
cudaError_t set_attrs() {
  cudaError_t e;
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
  if ((e = set_attrs<T, 256, 128, 4>()) != cudaSuccess) return e;
  // Two K blocks per stage (3-D boxes) for the split-K tiles of 128 W rows.
  if ((e = set_attrs_kps2<T, false>()) != cudaSuccess) return e;
  if ((e = set_attrs_kps2<T, true>()) != cudaSuccess) return e;
  if ((e = set_attrs_raw<T, kRawW>()) != cudaSuccess) return e;
  if ((e = set_attrs_raw<T, kRawA>()) != cudaSuccess) return e;
  return set_attrs_raw<T, kRawW | kRawA>();
}

template <typename T, int BT, int TN, int STAGES, bool WMN, bool GATHER, int RAW = 0, int KPS = 1>
cudaError_t launch_typed(const Problem& p, int split, const Gather* g, unsigned int* err, cudaStream_t stream) {
  constexpr int64_t esz = 2;
  TmaSet<RAW> maps;
  RawClasses w_rc, a_rc;
  bool ok = true;
  bool w_3d = false;
  if constexpr ((RAW & kRawW) != 0) {
    // W rows TMA cannot address as they are: one unswizzled map per row class.
    ok = encode_raw(maps.w, Elem<T>::kTmaType, p.b, p.n, p.k, p.b_ns, TN, &w_rc);
  } else if constexpr (WMN) {
    // B = [K, N]: rows k (pitch b_ks), N contiguous; one 3-D box of
    // 64(n) x 64 * KPS(k) x TN / 64 column blocks when N is whole blocks of 64,
    // else TN / 64 boxes of 64(n) x 64(k).
    w_3d = KPS == 2 || p.n % 64 == 0;
    ok = w_3d ? encode_mn_3d(&maps.w[0], Elem<T>::kTmaType, p.b, p.n, p.k, p.b_ks * esz, kTileK * KPS, TN / 64)
              : encode_2d(&maps.w[0], Elem<T>::kTmaType, p.b, p.n, p.k, p.b_ks * esz, 64, kTileK);
  } else {
    // W = B^T: rows n (pitch b_ns), K contiguous; boxes 64(k) x TN (x 2 K blocks).
    const int64_t w_pitch = p.n > 1 ? p.b_ns * esz : ((p.k * esz + 15) / 16) * 16;
    ok = KPS == 2 ? encode_kblocks_3d(&maps.w[0], Elem<T>::kTmaType, p.b, p.k, p.n, w_pitch, TN)
                  : encode_2d(&maps.w[0], Elem<T>::kTmaType, p.b, p.k, p.n, w_pitch, kTileK, TN);
  }
  if constexpr ((RAW & kRawA) != 0) {
    ok = ok && encode_raw(maps.a, Elem<T>::kTmaType, p.a, p.m, p.k, p.a_rs, BT, &a_rc);
  } else {
    // A: rows m (pitch a_rs), K contiguous; boxes 64(k) x BT (x 2 K blocks).
    const int64_t a_pitch = p.m > 1 ? p.a_rs * esz : ((p.k * esz + 15) / 16) * 16;
    ok = ok && (KPS == 2 ? encode_kblocks_3d(&maps.a[0], Elem<T>::kTmaType, p.a, p.k, p.m, a_pitch, BT)
                         : encode_2d(&maps.a[0], Elem<T>::kTmaType, p.a, p.k, p.m, a_pitch, kTileK, BT));
  }
  if (!ok) return cudaErrorInvalidValue;
  using Cfg = TcConfig<BT, TN, STAGES, RAW, KPS>;
  // The raw boxes of the operands' row classes must fit their load-stage areas.
  if constexpr ((RAW & kRawW) != 0) {
    if (raw_class_offset(w_rc.classes, TN / w_rc.classes) > Cfg::kLoadWBytes) return cudaErrorInvalidValue;
  }
  if constexpr ((RAW & kRawA) != 0) {
    if (raw_class_offset(a_rc.classes, BT / a_rc.classes) > Cfg::kLoadABytes) return cudaErrorInvalidValue;
  }
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
  args.w_3d = w_3d ? 1 : 0;
  args.w_classes = w_rc.classes;
  args.w_shifts = w_rc.shifts;
  args.a_classes = a_rc.classes;
  args.a_shifts = a_rc.shifts;
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
  constexpr bool kPair = TN == 128 && BT <= 32 &&
                         STAGES == (KPS == 2 ? kPairStagesKps2 : RAW != 0 ? raw_pair_stages(RAW) : kPairStages);
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
  return cudaLaunchKernelEx(&cfg, tc_linear_kernel<T, BT, TN, STAGES, WMN, GATHER, RAW, KPS>, maps, args);
}

// Operands TMA cannot address as they are: the RAW kernels (128-row tiles).
template <typename T, int RAW>
cudaError_t launch_raw(const Problem& p, int split, int tile_t, int tile_n, int stages, unsigned int* err,
                       cudaStream_t s) {
  if (tile_n != 128) return cudaErrorInvalidValue;
  if (stages == kPairStages) {
    constexpr int kPair = raw_pair_stages(RAW);
    switch (tile_t) {
      case 16: return launch_typed<T, 16, 128, kPair, false, false, RAW>(p, split, nullptr, err, s);
      case 32: return launch_typed<T, 32, 128, kPair, false, false, RAW>(p, split, nullptr, err, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (tile_t) {
    case 16: return launch_typed<T, 16, 128, 8, false, false, RAW>(p, split, nullptr, err, s);
    case 32: return launch_typed<T, 32, 128, 8, false, false, RAW>(p, split, nullptr, err, s);
    case 64: return launch_typed<T, 64, 128, 6, false, false, RAW>(p, split, nullptr, err, s);
    case 128: return launch_typed<T, 128, 128, 4, false, false, RAW>(p, split, nullptr, err, s);
    case 256: return launch_typed<T, 256, 128, 2, false, false, RAW>(p, split, nullptr, err, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_raw_any(const Problem& p, int split, int tile_t, int tile_n, int stages, unsigned int* err,
                           cudaStream_t s) {
  switch (p.raw) {
    case kRawW: return launch_raw<T, kRawW>(p, split, tile_t, tile_n, stages, err, s);
    case kRawA: return launch_raw<T, kRawA>(p, split, tile_t, tile_n, stages, err, s);
    case kRawW | kRawA: return launch_raw<T, kRawW | kRawA>(p, split, tile_t, tile_n, stages, err, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, bool WMN, bool GATHER>
cudaError_t launch_bt(const Problem& p, int split, int tile_t, int tile_n, int stages, int kps, const Gather* g,
                      unsigned int* err, cudaStream_t s) {
  if (kps == 2) {
    if (tile_n != 128 || stages != kps2_stages(tile_t, stages == kPairStagesKps2)) return cudaErrorInvalidValue;
    switch (tile_t) {
      case 16: return launch_typed<T, 16, 128, kPairStagesKps2, WMN, GATHER, 0, 2>(p, split, g, err, s);
      case 32: return launch_typed<T, 32, 128, kPairStagesKps2, WMN, GATHER, 0, 2>(p, split, g, err, s);
      case 64: return launch_typed<T, 64, 128, 4, WMN, GATHER, 0, 2>(p, split, g, err, s);
      case 128: return launch_typed<T, 128, 128, 3, WMN, GATHER, 0, 2>(p, split, g, err, s);
      default: return cudaErrorInvalidValue;
    }
  }
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

cudaError_t launch_tc(const Problem& p, int split, int tile_t, int tile_n, int stages, int kps, int w_mn,
                      const Gather* g, unsigned int* err, cudaStream_t s) {
  if (p.raw != 0) {
    if (g != nullptr || w_mn) return cudaErrorInvalidValue;
    return p.dtype == GLQ_DTYPE_BF16 ? launch_raw_any<__nv_bfloat16>(p, split, tile_t, tile_n, stages, err, s)
                                     : launch_raw_any<__half>(p, split, tile_t, tile_n, stages, err, s);
  }
  if (g != nullptr) {
    if (p.dtype == GLQ_DTYPE_BF16) {
      return w_mn ? launch_bt<__nv_bfloat16, true, true>(p, split, tile_t, tile_n, stages, kps, g, err, s)
                  : launch_bt<__nv_bfloat16, false, true>(p, split, tile_t, tile_n, stages, kps, g, err, s);
    }
    return w_mn ? launch_bt<__half, true, true>(p, split, tile_t, tile_n, stages, kps, g, err, s)
                : launch_bt<__half, false, true>(p, split, tile_t, tile_n, stages, kps, g, err, s);
  }
  if (p.dtype == GLQ_DTYPE_BF16) {
    return w_mn ? launch_bt<__nv_bfloat16, true, false>(p, split, tile_t, tile_n, stages, kps, g, err, s)
                : launch_bt<__nv_bfloat16, false, false>(p, split, tile_t, tile_n, stages, kps, g, err, s);
  }
  return w_mn ? launch_bt<__half, true, false>(p, split, tile_t, tile_n, stages, kps, g, err, s)
              : launch_bt<__half, false, false>(p, split, tile_t, tile_n, stages, kps, g, err, s);
}

}  // namespace glq
