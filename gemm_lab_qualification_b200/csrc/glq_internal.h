// glq_internal.h -- declarations shared by the kernel translation units and
// the C-ABI layer of libglq.so.  Not installed; include/glq.h is the public
// surface.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/glq.h"

namespace glq {

// Bits of the per-device sticky error word (glq_device_error).
enum DeviceErrorBits : unsigned int {
  kErrTimeoutProducer = 1u << 0,  // TMA producer gave up waiting for a free stage
  kErrTimeoutMma = 1u << 1,       // MMA issuer gave up waiting for a filled stage
  kErrTimeoutEpilogue = 1u << 2,  // epilogue gave up waiting for the accumulator
  kErrTimeoutDrain = 1u << 3,     // in-flight TMA loads did not land at exit
  kErrSmemAlign = 1u << 4,        // dynamic shared memory not 1024-B aligned
  kErrTimeoutPeer = 1u << 5,      // a peer rank never published its gathered slice
};

// Time budget of one bounded in-kernel wait.  Legitimate waits last
// microseconds; this only ends a wait that can no longer complete.
constexpr uint64_t kWaitBudgetNs = 1000ull * 1000ull * 1000ull;  // 1 s

// One linear problem after argument validation.  Strides in elements.
struct Problem {
  int dtype;  // glq_dtype
  const void* a;
  int64_t a_rs, a_cs;
  const void* b;
  int64_t b_ks, b_ns;
  const void* bias;
  int epilogue;  // glq_epilogue
  void* y;
  int64_t ldy;
  int64_t m, n, k;
  float* partial;  // optional [split, m, n] FP32 split partials
  unsigned int flags;  // glq_flags
  int require_tc;      // 1: the tcgen05 kernel or an error (fused gather)
  int raw;             // kRawW | kRawA: operands the tcgen05 kernel stages raw and aligns itself
};

// Fused all-gather of a column-parallel layer (glq_linear_gather): output
// bases already offset to this rank's first column, and the completion
// protocol's signal slots.
struct Gather {
  int rank, world;
  void* y[GLQ_MAX_RANKS];
  unsigned long long* signal[GLQ_MAX_RANKS];
  unsigned int* counter;
  unsigned long long epoch;
};

// Operands of the tcgen05 kernel that TMA cannot address as they are
// (K-contiguous rows with a base or row pitch off 16 bytes): the kernel
// loads them by row class and aligns them in shared memory.
constexpr int kRawW = 1;
constexpr int kRawA = 2;
// Row classes of a raw operand: rows r == c (mod C) share one tensor map.
constexpr int kMaxClasses = 8;

// Row pitch (elements) the row classes are computed from: a single row has
// no pitch, any multiple of 8 past its end serves.
inline int64_t raw_pitch(int64_t rows, int64_t k, int64_t pitch) {
  return rows <= 1 ? (k + 15) / 8 * 8 : pitch;
}

// Class count C (power of two, at most kMaxClasses) and the per-class
// element offsets s_c (4 bits each) of a raw operand: rows x k, K
// contiguous, row pitch `pitch` elements, base 2-byte aligned.  C * pitch
// must be a multiple of 8 elements (16 bytes: a TMA row pitch) and at least
// k + 8 (a class's rows, each read as k + s_c <= k + 7 elements, do not
// overlap); false when no C <= kMaxClasses satisfies both.
struct RawClasses {
  int classes = 1;
  unsigned int shifts = 0;
};
inline bool raw_classes(const void* base, int64_t rows, int64_t k, int64_t pitch, RawClasses* out) {
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  if ((b & 1u) != 0 || rows <= 0 || k <= 0) return false;
  const int64_t pe = raw_pitch(rows, k, pitch);
  if (pe < k) return false;
  int c = pe % 8 == 0 ? 1 : pe % 4 == 0 ? 2 : pe % 2 == 0 ? 4 : 8;
  while (c < kMaxClasses && c * pe < k + 8) c *= 2;
  if (c * pe < k + 8) return false;
  const int64_t b0 = static_cast<int64_t>((b & 15u) >> 1);
  out->classes = c;
  out->shifts = 0;
  for (int i = 0; i < c; ++i) out->shifts |= static_cast<unsigned int>((b0 + i * pe) & 7) << (4 * i);
  return true;
}

// How the operands sit in memory: unit-stride dimensions and whether the
// TMA kernels can address them (16-byte aligned bases and row pitches, rows
// that do not overlap).
struct OperandLayout {
  bool a_unit = false, a_ok = false;
  bool w_kmajor = false, w_mnmajor = false, w_ok = false;
};
OperandLayout classify(const Problem& p);

// Copies of the operands the TMA kernels cannot address, in a caller
// workspace: A first ([M, K], K-contiguous), then W (K-contiguous [N, K],
// or [K, N] when B is N-contiguous), each 256-byte aligned.
struct RepackPlan {
  bool a = false, w = false, w_mn = false;
  size_t a_bytes = 0, w_bytes = 0;
  size_t bytes() const { return a_bytes + w_bytes; }
};
// kRawW / kRawA bits when the tcgen05 kernel can run with the operands that
// TMA cannot address staged raw and aligned in shared memory (K-contiguous
// rows, W K-major, row classes as raw_classes), 0 when both operands are
// addressable, -1 when the problem needs the small or generic kernel or
// aligned copies.
int raw_operands(const Problem& p, const OperandLayout& L);
// False when every operand is already TMA-addressable (or nothing to do).
bool repack_plan(const Problem& p, RepackPlan* r);
// The same problem reading the copies in `workspace`.
Problem repacked_problem(const Problem& p, const RepackPlan& r, void* workspace);
cudaError_t launch_repacks(const Problem& p, const RepackPlan& r, void* workspace, int sm_count, cudaStream_t s);

// Path selection result.
struct Choice {
  int path;     // glq_path
  int split;    // K ranges merged in-kernel (1 = none)
  int kernel;   // Kernel below
  int tile_t;   // token tile (MMA N) of the tcgen05 kernel
  int tile_n;   // W rows per CTA of the tcgen05 kernel (128 or 256)
  int stages;   // TMA ring depth of the tcgen05 kernel (kPairStages: two CTAs per SM)
  int kps;      // K blocks per TMA stage of the tcgen05 kernel (1, or 2 with 3-D boxes)
  int w_mn;     // 1: W = B^T is N-contiguous (B = [K, N]); MN-major W tiles
  int raw;      // kRawW | kRawA: operands staged raw and aligned by the tcgen05 kernel (path tc_ldg)
};

enum Kernel : int {
  kKernelNone = 0,
  kKernelFill = 1,
  kKernelGemv = 2,
  kKernelTc = 3,
  kKernelGeneric = 4,
  kKernelGemvRing = 5,  // M = 1 GEMV fed by the TMA engine (path gemv_m1)
  kKernelSmall = 6,     // few multiply-adds, any layout: K spread over warps
};

// Pure host planning (glq_plan and glq_linear share it).
int plan_problem(const Problem& p, int split_k, int sm_count, Choice* out);

// Number of 64-wide K blocks of the tcgen05 kernel.
inline int64_t tc_k_blocks(int64_t k) { return (k + 63) / 64; }

// W rows per CTA of the tcgen05 kernel: 256-row tiles (32 KB TMA boxes) for
// small token tiles when the layer is wide enough to fill the device with at
// most 4-way split-K (N >= 8192), 128 otherwise.
inline int tc_tile_rows(int64_t m, int64_t n) { return (m <= 32 && n >= 8192) ? 256 : 128; }

// Largest automatic split-K: clusters of up to 4 CTAs with ~200 KB of shared
// memory each still pack one wave onto the 148 SMs (33 clusters of 4 are
// co-resident on B200); larger clusters may not, which costs a second wave.
constexpr int kMaxAutoSplit = 4;

// Small token tiles on narrow layers: two CTAs per SM (4-stage ring plus a
// dedicated split-K receive buffer, under 113 KB of shared memory), so an
// 8-way split-K cluster still packs one wave (33 clusters of 8 are
// co-resident at that size).
constexpr int kPairSplit = 8;
constexpr int kPairStages = 4;
// The same split with two K blocks per stage: one 32 KB W box (and one A
// box) per TMA operation, two stages (the same bytes in flight).
constexpr int kPairStagesKps2 = 2;
constexpr int kPairKps = 2;  // K blocks per stage the planner picks for that split when K allows
// Ring depth of the two-K-blocks-per-stage kernels (half the one-block
// depth, the same bytes in flight): the two-CTAs-per-SM split, and the
// one-CTA-per-SM split-K tiles of 64 and 128 tokens; 0 where there is none.
inline int kps2_stages(int tile_t, bool pair) {
  if (pair) return tile_t <= 32 ? kPairStagesKps2 : 0;
  return tile_t == 64 ? 4 : tile_t == 128 ? 3 : 0;
}

// Operands the tcgen05 kernel can stage raw and align itself are copied
// instead when the caller gives a repack workspace and the problem has more
// than this many tokens: every token tile re-aligns the same W tiles, where
// one copy serves them all (509 x 4099 x 4103: 103 us aligned in shared
// memory, 56 us copied).
constexpr int64_t kRawCopyAboveTokens = 128;

// Token tile of the tcgen05 kernel for m tokens.
inline int tc_token_tile(int64_t m) {
  if (m <= 16) return 16;
  if (m <= 32) return 32;
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

// Launchers (return cudaError_t of the launch).  err = device error word.
cudaError_t launch_fill(const Problem& p, cudaStream_t s);
cudaError_t launch_gemv(const Problem& p, int split, unsigned int* err, cudaStream_t s);
cudaError_t launch_gemv_ring(const Problem& p, unsigned int* err, cudaStream_t s, int sm_count);

// Where the ring GEMV runs: rows of at most 8 KB (K <= 4096, K % 8 == 0)
// and at most 32 rows per SM, i.e. layers the register GEMV covers in one
// wave, so the whole weight can be requested at once.  Taller layers stream
// better through the register GEMV's successive waves (measured: 28672 x 8192
// 73 us register GEMV vs 136 us ring), and the ring's shared memory (A, the
// per-row partials and at least two stages) must fit in 227 KB.
inline bool gemv_ring_fits(int64_t n, int64_t k, int sm_count) {
  if (k % 8 != 0 || k <= 0 || k > 4096 || n <= 0) return false;
  const int64_t ctas = n < sm_count ? n : sm_count;
  const int64_t rows = (n + ctas - 1) / ctas;
  if (rows > 32) return false;
  const int64_t fixed = 2 * k + ((rows * 4 + 15) / 16) * 16 + 1024;
  return fixed + 2 * k * 2 <= 232448;
}
cudaError_t launch_generic(const Problem& p, cudaStream_t s);
// Strided or unaligned problems of at most this many multiply-adds run the
// small kernel: its latency is a few memory round trips, where the tiled
// generic kernel walks K in sequence and a repack costs extra launches.
constexpr int64_t kSmallMacs = int64_t(1) << 22;
inline bool small_problem(int64_t m, int64_t n, int64_t k) {
  return m > 0 && n > 0 && k > 0 && m <= 65535 && m * n <= kSmallMacs && m * n * k <= kSmallMacs;
}
cudaError_t launch_small(const Problem& p, cudaStream_t s);

// Row pitch (elements) of a repacked operand: rows start on 16-byte
// boundaries.
inline int64_t repack_pitch(int64_t cols) { return (cols + 7) / 8 * 8; }
// Copies rows x cols 2-byte elements, element (r, c) at src + r*rs + c*cs
// (any alignment), into dst (16-byte aligned) with row pitch
// repack_pitch(cols); the pad columns are written as zero.
cudaError_t launch_repack(const void* src, int64_t rows, int64_t cols, int64_t rs, int64_t cs, void* dst,
                          int sm_count, cudaStream_t s);
// Returns cudaErrorNotSupported-style codes through `status` for TMA encode
// problems (GLQ_ERR_CUDA).
// gather: null for a plain call (the output is p.y only).
// kps: K blocks per load stage (2: 3-D TMA boxes of two K blocks, the
// two-CTAs-per-SM split with stages == kPairStagesKps2).
cudaError_t launch_tc(const Problem& p, int split, int tile_t, int tile_n, int stages, int kps, int w_mn,
                      const Gather* gather, unsigned int* err, cudaStream_t s);

// Per-device one-time set-up of the tcgen05 kernels (shared memory opt-in).
cudaError_t tc_prepare_device();
// ... and of the ring GEMV.
cudaError_t gemv_prepare_device();

}  // namespace glq
