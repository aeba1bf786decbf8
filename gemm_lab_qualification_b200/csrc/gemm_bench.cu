// gemm_bench.cu -- native benchmark CLI for libglq.so (sm_100a).
//
// Command-line surface of the lab's native benchmark (flags
// csrc/gemm_bench.cu:321-345, JSON schema v1 csrc/gemm_bench.cu:1274-1323,
// exit status 0 = pass, 1 = any error including a failed correctness gate),
// with this library's kernels as --impl names next to the two vendor
// references:
//
//   cublas      cublasGemmEx, FP32 compute (spot-checked against CPU FP64)
//   cublaslt    cublasLtMatmul with the heuristic's first algorithm
//   glq         glq_matmul: the lab's B = [K, N] operand as given
//   glq_splitk  glq_splitk_matmul: K split merged in-kernel, FP32 partials
//               written to a caller workspace (the lab's split-K contract)
//   glq_wnk     glq_linear with the weight stored K-contiguous (W = B^T,
//               transposed once before timing): a linear layer's layout
//
// C = A . B with A [M, K], B [K, N], C [M, N] row-major, FP32 accumulation.
// Every glq implementation is checked element by element against cuBLAS
// before anything is timed; a failure exits 1 without timing.
#include <cublasLt.h>
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <memory>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "glq.h"

namespace {

// ------------------------------------------------------------------ errors

void cuda_ok(cudaError_t e, const char* what, int line) {
  if (e != cudaSuccess) {
    std::ostringstream s;
    s << what << " (gemm_bench.cu:" << line << "): " << cudaGetErrorString(e);
    throw std::runtime_error(s.str());
  }
}
#define CUDA_OK(x) cuda_ok((x), #x, __LINE__)

void cublas_ok(cublasStatus_t st, const char* what, int line) {
  if (st != CUBLAS_STATUS_SUCCESS) {
    std::ostringstream s;
    s << what << " (gemm_bench.cu:" << line << "): cuBLAS status " << static_cast<int>(st);
    throw std::runtime_error(s.str());
  }
}
#define CUBLAS_OK(x) cublas_ok((x), #x, __LINE__)

void glq_ok(int st, const char* what) {
  if (st != GLQ_OK) throw std::runtime_error(std::string(what) + ": " + glq_status_string(st));
}

// ------------------------------------------------------------------ options

struct Options {
  int64_t m = 512, n = 512, k = 512;
  std::string dtype = "fp16";
  std::string impl = "cublas";
  std::string cache = "steady";
  int warmup = 25;
  double warmup_seconds = 0.0;
  int samples = 100;
  double measurement_seconds = 0.0;
  double min_sample_ms = 0.25;
  int max_inner = 100;
  int seed = 17;
  int correctness_samples = 64;
  int split_k = 0;
  bool pretty = false;
};

const char* kUsage =
    "gemm_bench -- B200 (sm_100a) linear-fragment benchmark\n\n"
    "Usage: gemm_bench [options]\n\n"
    "  --m INT                    rows of A and C (default 512)\n"
    "  --n INT                    columns of B and C (default 512)\n"
    "  --k INT                    reduction length (default 512)\n"
    "  --dtype fp16|bf16|fp32     element type; glq_* take fp16 and bf16 (default fp16)\n"
    "  --impl cublas|cublaslt|glq|glq_splitk|glq_wnk   (default cublas)\n"
    "  --cache steady|cold        cold writes a 2 x L2 buffer before every sample (default steady)\n"
    "  --warmup INT               warm-up launches (default 25)\n"
    "  --warmup-seconds NUMBER    minimum warm-up time (default 0)\n"
    "  --samples INT              timed samples (default 100)\n"
    "  --measurement-seconds NUM  minimum timed duration (default 0)\n"
    "  --min-sample-ms NUM        steady cache: launches per sample until one sample lasts this long\n"
    "                             (default 0.25)\n"
    "  --max-inner-repetitions N  cap on launches per sample (default 100)\n"
    "  --seed INT                 input seed (default 17)\n"
    "  --correctness-samples INT  CPU FP64 spot checks of the vendor references (default 64)\n"
    "  --split-k INT              glq_splitk: number of K ranges (0 = the library's choice)\n"
    "  --pretty                   indented JSON\n"
    "  --help                     this text\n";

int64_t to_int(const std::string& flag, const std::string& v, int64_t max_value) {
  size_t used = 0;
  long long x = 0;
  try {
    x = std::stoll(v, &used);
  } catch (const std::exception&) {
    throw std::invalid_argument(flag + " needs an integer, got '" + v + "'");
  }
  if (used != v.size() || x < 0 || x > max_value) {
    throw std::invalid_argument(flag + " needs an integer in 0.." + std::to_string(max_value) + ", got '" + v + "'");
  }
  return x;
}

double to_number(const std::string& flag, const std::string& v) {
  size_t used = 0;
  double x = 0.0;
  try {
    x = std::stod(v, &used);
  } catch (const std::exception&) {
    throw std::invalid_argument(flag + " needs a number, got '" + v + "'");
  }
  if (used != v.size() || !std::isfinite(x) || x < 0.0) {
    throw std::invalid_argument(flag + " needs a finite number >= 0, got '" + v + "'");
  }
  return x;
}

Options parse(int argc, char** argv) {
  Options o;
  constexpr int64_t kIntMax = 2147483647;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--help") {
      std::cout << kUsage;
      std::exit(0);
    }
    if (a == "--pretty") {
      o.pretty = true;
      continue;
    }
    if (i + 1 >= argc) throw std::invalid_argument("no value after " + a);
    const std::string v = argv[++i];
    if (a == "--m") o.m = to_int(a, v, kIntMax);
    else if (a == "--n") o.n = to_int(a, v, kIntMax);
    else if (a == "--k") o.k = to_int(a, v, kIntMax);
    else if (a == "--dtype") o.dtype = v;
    else if (a == "--impl") o.impl = v;
    else if (a == "--cache") o.cache = v;
    else if (a == "--warmup") o.warmup = static_cast<int>(to_int(a, v, kIntMax));
    else if (a == "--warmup-seconds") o.warmup_seconds = to_number(a, v);
    else if (a == "--samples") o.samples = static_cast<int>(to_int(a, v, kIntMax));
    else if (a == "--measurement-seconds") o.measurement_seconds = to_number(a, v);
    else if (a == "--min-sample-ms") o.min_sample_ms = to_number(a, v);
    else if (a == "--max-inner-repetitions") o.max_inner = static_cast<int>(to_int(a, v, kIntMax));
    else if (a == "--seed") o.seed = static_cast<int>(to_int(a, v, kIntMax));
    else if (a == "--correctness-samples") o.correctness_samples = static_cast<int>(to_int(a, v, kIntMax));
    else if (a == "--split-k") o.split_k = static_cast<int>(to_int(a, v, GLQ_MAX_SPLIT));
    else throw std::invalid_argument("unknown option " + a + " (see --help)");
  }
  if (o.dtype != "fp16" && o.dtype != "bf16" && o.dtype != "fp32") {
    throw std::invalid_argument("--dtype must be fp16, bf16 or fp32");
  }
  const bool ours = o.impl == "glq" || o.impl == "glq_splitk" || o.impl == "glq_wnk";
  if (!ours && o.impl != "cublas" && o.impl != "cublaslt") {
    throw std::invalid_argument("--impl must be cublas, cublaslt, glq, glq_splitk or glq_wnk");
  }
  if (ours && o.dtype == "fp32") throw std::invalid_argument("the glq implementations take fp16 or bf16");
  if (o.cache != "steady" && o.cache != "cold") throw std::invalid_argument("--cache must be steady or cold");
  if (o.m == 0 || o.n == 0 || o.k == 0) throw std::invalid_argument("--m, --n and --k must be positive");
  if (o.samples == 0) throw std::invalid_argument("--samples must be positive");
  if (o.max_inner == 0) throw std::invalid_argument("--max-inner-repetitions must be positive");
  if (o.correctness_samples == 0) throw std::invalid_argument("--correctness-samples must be positive");
  return o;
}

// ------------------------------------------------------------------ element types

template <typename T> struct Type;
template <> struct Type<float> {
  static constexpr cudaDataType_t kCuda = CUDA_R_32F;
  static constexpr int kGlq = -1;
  static float to(float v) { return v; }
  static float from(float v) { return v; }
  static const char* name() { return "float32"; }
  static double atol() { return 1.0e-4; }
  static double rtol() { return 1.0e-4; }
};
template <> struct Type<__half> {
  static constexpr cudaDataType_t kCuda = CUDA_R_16F;
  static constexpr int kGlq = GLQ_DTYPE_F16;
  static __half to(float v) { return __float2half_rn(v); }
  static float from(__half v) { return __half2float(v); }
  static const char* name() { return "float16"; }
  static double atol() { return 2.0e-2; }
  static double rtol() { return 2.0e-2; }
};
template <> struct Type<__nv_bfloat16> {
  static constexpr cudaDataType_t kCuda = CUDA_R_16BF;
  static constexpr int kGlq = GLQ_DTYPE_BF16;
  static __nv_bfloat16 to(float v) { return __float2bfloat16_rn(v); }
  static float from(__nv_bfloat16 v) { return __bfloat162float(v); }
  static const char* name() { return "bfloat16"; }
  static double atol() { return 8.0e-2; }
  static double rtol() { return 5.0e-2; }
};

// Deterministic inputs: uniform [-0.25, 0.25) per (seed, operand).
template <typename T>
std::vector<T> inputs(size_t count, int seed, int operand) {
  std::seed_seq seq{seed, operand, 0x51ed};
  std::mt19937_64 gen(seq);
  std::uniform_real_distribution<float> dist(-0.25f, 0.25f);
  std::vector<T> v(count);
  for (auto& x : v) x = Type<T>::to(dist(gen));
  return v;
}

// ------------------------------------------------------------------ device memory

struct DeviceMem {
  void* p = nullptr;
  size_t bytes = 0;
  DeviceMem() = default;
  explicit DeviceMem(size_t b) : bytes(b) {
    if (b) CUDA_OK(cudaMalloc(&p, b));
  }
  ~DeviceMem() {
    if (p) cudaFree(p);
  }
  DeviceMem(const DeviceMem&) = delete;
  DeviceMem& operator=(const DeviceMem&) = delete;
  DeviceMem(DeviceMem&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DeviceMem& operator=(DeviceMem&& o) noexcept {
    std::swap(p, o.p);
    std::swap(bytes, o.bytes);
    return *this;
  }
  template <typename T> T* as() const { return static_cast<T*>(p); }
};

__global__ void scribble(uint32_t* buf, size_t words, uint32_t salt) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    buf[i] = static_cast<uint32_t>(i) ^ salt;
  }
}

// out[n][k] = in[k][n] (one-off layout change before timing)
template <typename T>
__global__ void transpose(const T* in, T* out, int64_t rows, int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    out[c * rows + r] = in[i];
  }
}

// ------------------------------------------------------------------ implementations

struct LtPlan {
  cublasLtHandle_t handle = nullptr;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulAlgo_t algo{};
  DeviceMem workspace;
  size_t ws_bytes = 0;

  // Row-major C = A B is column-major C^T = B^T A^T: the library's "A" is B
  // (n x k, ld n), its "B" is A (k x m, ld k), C is n x m (ld n).
  LtPlan(cudaDataType_t t, int64_t m, int64_t n, int64_t k) {
    CUBLAS_OK(cublasLtCreate(&handle));
    const cublasComputeType_t compute = t == CUDA_R_32F ? CUBLAS_COMPUTE_32F_PEDANTIC : CUBLAS_COMPUTE_32F;
    CUBLAS_OK(cublasLtMatmulDescCreate(&op, compute, CUDA_R_32F));
    CUBLAS_OK(cublasLtMatrixLayoutCreate(&la, t, n, k, n));
    CUBLAS_OK(cublasLtMatrixLayoutCreate(&lb, t, k, m, k));
    CUBLAS_OK(cublasLtMatrixLayoutCreate(&lc, t, n, m, n));
    cublasLtMatmulPreference_t pref = nullptr;
    CUBLAS_OK(cublasLtMatmulPreferenceCreate(&pref));
    const size_t max_ws = 32ull << 20;
    CUBLAS_OK(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &max_ws,
                                                   sizeof(max_ws)));
    cublasLtMatmulHeuristicResult_t result{};
    int found = 0;
    const cublasStatus_t st = cublasLtMatmulAlgoGetHeuristic(handle, op, la, lb, lc, lc, pref, 1, &result, &found);
    cublasLtMatmulPreferenceDestroy(pref);
    CUBLAS_OK(st);
    if (found == 0) throw std::runtime_error("cuBLASLt found no algorithm for this shape");
    algo = result.algo;
    ws_bytes = result.workspaceSize;
    workspace = DeviceMem(ws_bytes);
  }
  ~LtPlan() {
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (op) cublasLtMatmulDescDestroy(op);
    if (handle) cublasLtDestroy(handle);
  }
  void run(const void* a, const void* b, void* c, cudaStream_t s) {
    const float one = 1.0f, zero = 0.0f;
    CUBLAS_OK(cublasLtMatmul(handle, op, &one, b, la, a, lb, &zero, c, lc, c, lc, &algo, workspace.p, ws_bytes, s));
  }
};

template <typename T>
void cublas_gemm(cublasHandle_t h, const T* a, const T* b, T* c, int64_t m, int64_t n, int64_t k) {
  const float one = 1.0f, zero = 0.0f;
  const cublasComputeType_t compute =
      std::is_same<T, float>::value ? CUBLAS_COMPUTE_32F_PEDANTIC : CUBLAS_COMPUTE_32F;
  CUBLAS_OK(cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, static_cast<int>(n), static_cast<int>(m), static_cast<int>(k),
                         &one, b, Type<T>::kCuda, static_cast<int>(n), a, Type<T>::kCuda, static_cast<int>(k), &zero, c,
                         Type<T>::kCuda, static_cast<int>(n), compute, CUBLAS_GEMM_DEFAULT));
}

// ------------------------------------------------------------------ checks and statistics

struct Check {
  bool passed = true;
  std::string reference;
  double atol = 0, rtol = 0, max_abs = 0, max_rel = 0, l2 = 0;
  int64_t nan = 0, inf = 0, checked = 0;
};

template <typename T>
Check compare(const std::vector<double>& got, const std::vector<double>& want, const std::string& reference) {
  Check c;
  c.reference = reference;
  c.atol = Type<T>::atol();
  c.rtol = Type<T>::rtol();
  double err2 = 0, ref2 = 0;
  for (size_t i = 0; i < got.size(); ++i) {
    ++c.checked;
    if (std::isnan(got[i])) { ++c.nan; c.passed = false; continue; }
    if (std::isinf(got[i])) { ++c.inf; c.passed = false; continue; }
    const double e = std::fabs(got[i] - want[i]);
    c.max_abs = std::max(c.max_abs, e);
    c.max_rel = std::max(c.max_rel, e / std::max(std::fabs(want[i]), 1e-12));
    err2 += e * e;
    ref2 += want[i] * want[i];
    if (e > c.atol + c.rtol * std::fabs(want[i])) c.passed = false;
  }
  c.l2 = std::sqrt(err2) / std::max(std::sqrt(ref2), 1e-12);
  return c;
}

struct Stats {
  double p05, p50, p95, mean, stddev, mad, cv;
};

Stats summarize(std::vector<double> ms) {
  std::sort(ms.begin(), ms.end());
  auto pick = [&](double q) { return ms[static_cast<size_t>(std::llround(q * static_cast<double>(ms.size() - 1)))]; };
  Stats s{};
  s.p05 = pick(0.05);
  s.p50 = pick(0.50);
  s.p95 = pick(0.95);
  double sum = 0;
  for (double x : ms) sum += x;
  s.mean = sum / static_cast<double>(ms.size());
  double var = 0;
  for (double x : ms) var += (x - s.mean) * (x - s.mean);
  s.stddev = ms.size() > 1 ? std::sqrt(var / static_cast<double>(ms.size() - 1)) : 0.0;
  std::vector<double> dev(ms.size());
  for (size_t i = 0; i < ms.size(); ++i) dev[i] = std::fabs(ms[i] - s.p50);
  std::sort(dev.begin(), dev.end());
  s.mad = dev[dev.size() / 2];
  s.cv = s.mean > 0 ? s.stddev / s.mean : 0.0;
  return s;
}

// ------------------------------------------------------------------ run

template <typename T>
int run(const Options& o) {
  const size_t na = static_cast<size_t>(o.m * o.k), nb = static_cast<size_t>(o.k * o.n),
               nc = static_cast<size_t>(o.m * o.n);
  const std::vector<T> ha = inputs<T>(na, o.seed, 1);
  const std::vector<T> hb = inputs<T>(nb, o.seed, 2);

  cudaStream_t stream = nullptr;
  CUDA_OK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  cublasHandle_t blas = nullptr;
  CUBLAS_OK(cublasCreate(&blas));
  CUBLAS_OK(cublasSetStream(blas, stream));
  CUBLAS_OK(cublasSetMathMode(blas, std::is_same<T, float>::value ? CUBLAS_PEDANTIC_MATH : CUBLAS_DEFAULT_MATH));

  DeviceMem da(na * sizeof(T)), db(nb * sizeof(T)), dc(nc * sizeof(T));
  CUDA_OK(cudaMemcpy(da.p, ha.data(), da.bytes, cudaMemcpyHostToDevice));
  CUDA_OK(cudaMemcpy(db.p, hb.data(), db.bytes, cudaMemcpyHostToDevice));

  int dev = 0, l2 = 0;
  CUDA_OK(cudaGetDevice(&dev));
  CUDA_OK(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
  DeviceMem evict(std::max<size_t>(2ull * static_cast<size_t>(l2), 32ull << 20));

  // Implementation set-up (never inside the timed region).
  std::unique_ptr<LtPlan> lt;
  DeviceMem partial, wnk, repack;
  int run_path = -1, run_split = 0;  // what the repacked launches report
  int splits = 1, path = -1, plan_split = 1;
  if (o.impl == "cublaslt") lt = std::make_unique<LtPlan>(Type<T>::kCuda, o.m, o.n, o.k);
  if (o.impl == "glq" || o.impl == "glq_splitk") {
    glq_ok(glq_plan(Type<T>::kGlq, da.p, o.k, 1, db.p, o.n, 1, o.n, o.m, o.n, o.k, o.split_k, 0, &path, &plan_split),
           "glq_plan");
    if (o.impl == "glq_splitk") {
      splits = o.split_k > 0 ? o.split_k : plan_split;
      glq_ok(glq_plan(Type<T>::kGlq, da.p, o.k, 1, db.p, o.n, 1, o.n, o.m, o.n, o.k, splits, 0, &path, &plan_split),
             "glq_plan");
      splits = plan_split;
      if (splits > 1) partial = DeviceMem(static_cast<size_t>(splits) * nc * sizeof(float));
    }
  }
  if (o.impl == "glq_wnk") {
    wnk = DeviceMem(nb * sizeof(T));
    transpose<T><<<1024, 256, 0, stream>>>(db.as<T>(), wnk.as<T>(), o.k, o.n);
    CUDA_OK(cudaGetLastError());
    glq_ok(glq_plan(Type<T>::kGlq, da.p, o.k, 1, wnk.p, 1, o.k, o.n, o.m, o.n, o.k, 0, 0, &path, &plan_split),
           "glq_plan");
  }
  // Row pitches that are not a multiple of 16 bytes (odd K or N): the
  // library copies the operands into aligned rows in this workspace and runs
  // the tensor-core kernels (path "repacked") instead of the generic kernel.
  if (o.impl == "glq" || o.impl == "glq_wnk") {
    const bool kn = o.impl == "glq";
    const size_t need = glq_linear_workspace_bytes(Type<T>::kGlq, da.p, o.k, 1, kn ? db.p : wnk.p, kn ? o.n : 1,
                                                   kn ? 1 : o.k, o.m, o.n, o.k);
    if (need) {
      repack = DeviceMem(need);
      path = GLQ_PATH_REPACKED;
    }
  }

  auto launch = [&]() {
    if (o.impl == "cublas") {
      cublas_gemm<T>(blas, da.as<T>(), db.as<T>(), dc.as<T>(), o.m, o.n, o.k);
    } else if (o.impl == "cublaslt") {
      lt->run(da.p, db.p, dc.p, stream);
    } else if constexpr (!std::is_same<T, float>::value) {
      const int g = Type<T>::kGlq;
      if (o.impl == "glq" && repack.p != nullptr) {
        glq_ok(glq_linear(g, da.p, o.k, 1, db.p, o.n, 1, nullptr, GLQ_EPILOGUE_NONE, dc.p, o.n, o.m, o.n, o.k, 0,
                          repack.p, repack.bytes, stream, &run_path, &run_split),
               "glq_linear");
      } else if (o.impl == "glq") {
        glq_ok(glq_matmul(g, da.p, db.p, dc.p, static_cast<int>(o.m), static_cast<int>(o.n), static_cast<int>(o.k),
                          stream),
               "glq_matmul");
      } else if (o.impl == "glq_splitk") {
        glq_ok(glq_splitk_matmul(g, da.p, db.p, dc.p, static_cast<int>(o.m), static_cast<int>(o.n),
                                 static_cast<int>(o.k), partial.as<float>(), splits, stream),
               "glq_splitk_matmul");
      } else {
        glq_ok(glq_linear(g, da.p, o.k, 1, wnk.p, 1, o.k, nullptr, GLQ_EPILOGUE_NONE, dc.p, o.n, o.m, o.n, o.k, 0,
                          repack.p, repack.bytes, stream, &run_path, &run_split),
               "glq_linear");
      }
    }
  };

  // Correctness before timing: the glq kernels element by element against
  // cuBLAS, the vendor references at sampled elements against CPU FP64.
  launch();
  CUDA_OK(cudaStreamSynchronize(stream));
  if (repack.p != nullptr) {
    path = run_path;
    plan_split = run_split;
  }
  std::vector<T> hc(nc);
  CUDA_OK(cudaMemcpy(hc.data(), dc.p, dc.bytes, cudaMemcpyDeviceToHost));
  Check check;
  if (o.impl == "cublas" || o.impl == "cublaslt") {
    const int64_t count = std::min<int64_t>(o.correctness_samples, static_cast<int64_t>(nc));
    std::vector<double> got, want;
    for (int64_t s = 0; s < count; ++s) {
      const int64_t idx = count == 1 ? 0 : s * (static_cast<int64_t>(nc) - 1) / (count - 1);
      const int64_t r = idx / o.n, col = idx % o.n;
      double acc = 0;
      for (int64_t t = 0; t < o.k; ++t) {
        acc += static_cast<double>(Type<T>::from(ha[r * o.k + t])) * static_cast<double>(Type<T>::from(hb[t * o.n + col]));
      }
      got.push_back(Type<T>::from(hc[idx]));
      want.push_back(acc);
    }
    check = compare<T>(got, want, "cpu_fp64_spot");
  } else {
    DeviceMem dref(nc * sizeof(T));
    cublas_gemm<T>(blas, da.as<T>(), db.as<T>(), dref.as<T>(), o.m, o.n, o.k);
    CUDA_OK(cudaStreamSynchronize(stream));
    std::vector<T> href(nc);
    CUDA_OK(cudaMemcpy(href.data(), dref.p, dref.bytes, cudaMemcpyDeviceToHost));
    std::vector<double> got(nc), want(nc);
    for (size_t i = 0; i < nc; ++i) {
      got[i] = Type<T>::from(hc[i]);
      want[i] = Type<T>::from(href[i]);
    }
    check = compare<T>(got, want, "cublas_full");
  }
  unsigned int word = 0;
  if (o.impl.rfind("glq", 0) == 0) glq_ok(glq_device_error(&word, 1), "glq_device_error");
  if (!check.passed || word != 0) {
    throw std::runtime_error("correctness gate failed (max abs error " + std::to_string(check.max_abs) +
                             ", device error word " + std::to_string(word) + "): nothing was timed");
  }

  // Warm-up, launches-per-sample calibration, timed samples.
  int warmed = 0;
  const auto w0 = std::chrono::steady_clock::now();
  while (warmed < o.warmup ||
         std::chrono::duration<double>(std::chrono::steady_clock::now() - w0).count() < o.warmup_seconds) {
    launch();
    ++warmed;
    CUDA_OK(cudaStreamSynchronize(stream));
  }
  cudaEvent_t e0, e1;
  CUDA_OK(cudaEventCreate(&e0));
  CUDA_OK(cudaEventCreate(&e1));
  int inner = 1;
  if (o.cache == "steady" && o.min_sample_ms > 0) {
    CUDA_OK(cudaEventRecord(e0, stream));
    launch();
    CUDA_OK(cudaEventRecord(e1, stream));
    CUDA_OK(cudaEventSynchronize(e1));
    float probe = 0;
    CUDA_OK(cudaEventElapsedTime(&probe, e0, e1));
    if (probe > 0) inner = std::min(o.max_inner, std::max(1, static_cast<int>(std::ceil(o.min_sample_ms / probe))));
  }
  std::vector<double> ms;
  const auto t0 = std::chrono::steady_clock::now();
  uint32_t salt = 1;
  while (static_cast<int>(ms.size()) < o.samples ||
         std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() < o.measurement_seconds) {
    if (o.cache == "cold") {
      scribble<<<1184, 256, 0, stream>>>(evict.as<uint32_t>(), evict.bytes / 4, salt++);
      CUDA_OK(cudaGetLastError());
      CUDA_OK(cudaStreamSynchronize(stream));
    }
    CUDA_OK(cudaEventRecord(e0, stream));
    for (int i = 0; i < inner; ++i) launch();
    CUDA_OK(cudaEventRecord(e1, stream));
    CUDA_OK(cudaEventSynchronize(e1));
    float span = 0;
    CUDA_OK(cudaEventElapsedTime(&span, e0, e1));
    ms.push_back(static_cast<double>(span) / inner);
  }
  if (o.impl.rfind("glq", 0) == 0) {
    glq_ok(glq_device_error(&word, 1), "glq_device_error");
    if (word != 0) throw std::runtime_error("a bounded in-kernel wait expired while timing");
  }
  const Stats st = summarize(ms);

  cudaDeviceProp prop{};
  CUDA_OK(cudaGetDeviceProperties(&prop, dev));
  int rt = 0, drv = 0;
  CUDA_OK(cudaRuntimeGetVersion(&rt));
  CUDA_OK(cudaDriverGetVersion(&drv));
  const size_t ws_bytes = lt ? lt->ws_bytes : partial.bytes;
  const double tflops = 2.0 * static_cast<double>(o.m) * o.n * o.k / (st.p50 * 1e-3) / 1e12;
  // Algorithmic HBM bytes of one call: A, B and C each moved once.
  const double bytes = static_cast<double>(sizeof(T)) *
                       (static_cast<double>(o.m) * o.k + static_cast<double>(o.k) * o.n + static_cast<double>(o.m) * o.n);
  const double gbs = bytes / (st.p50 * 1e-3) / 1e9;

  const char* nl = o.pretty ? "\n" : "";
  const char* i1 = o.pretty ? "  " : "";
  std::ostringstream j;
  j.precision(10);
  j << '{' << nl << i1 << "\"schema_version\":1," << nl;
  j << i1 << "\"implementation\":{\"name\":\"" << o.impl << "\",\"version\":\"glq-sm100a-native-v1\"";
  if (path >= 0) j << ",\"path\":\"" << glq_path_name(path) << "\",\"split_k\":" << (o.impl == "glq_splitk" ? splits : plan_split);
  j << "}," << nl;
  j << i1 << "\"workload\":{\"m\":" << o.m << ",\"n\":" << o.n << ",\"k\":" << o.k << ",\"input_dtype\":\""
    << Type<T>::name() << "\",\"accumulator_dtype\":\"float32\",\"output_dtype\":\"" << Type<T>::name() << "\"},"
    << nl;
  j << i1 << "\"environment\":{\"gpu_name\":\"" << prop.name << "\",\"compute_capability\":\"" << prop.major << '.'
    << prop.minor << "\",\"l2_bytes\":" << l2 << ",\"cuda_runtime\":" << rt << ",\"cuda_driver\":" << drv << "},"
    << nl;
  j << i1 << "\"correctness\":{\"passed\":" << (check.passed ? "true" : "false") << ",\"reference\":\""
    << check.reference << "\",\"atol\":" << check.atol << ",\"rtol\":" << check.rtol
    << ",\"max_abs_error\":" << check.max_abs << ",\"max_relative_error\":" << check.max_rel
    << ",\"normalized_l2_error\":" << check.l2 << ",\"nan_count\":" << check.nan << ",\"inf_count\":" << check.inf
    << ",\"elements_checked\":" << check.checked << "}," << nl;
  j << i1 << "\"benchmark\":{\"cache_mode\":\"" << o.cache
    << "\",\"launch_mode\":\"eager\",\"timing_method\":\"cuda_event\",\"warmup_iterations\":" << warmed
    << ",\"warmup_min_seconds\":" << o.warmup_seconds << ",\"samples\":" << ms.size()
    << ",\"sample_inner_repetitions\":" << inner << ",\"measurement_min_seconds\":" << o.measurement_seconds
    << ",\"workspace_bytes\":" << ws_bytes << ",\"split_k\":" << splits << ",\"latency_ms\":{\"p05\":" << st.p05
    << ",\"p50\":" << st.p50 << ",\"p95\":" << st.p95 << ",\"mean\":" << st.mean << ",\"stddev\":" << st.stddev
    << ",\"mad\":" << st.mad << ",\"cv\":" << st.cv << "},\"tflops_p50\":" << tflops
    << ",\"algorithmic_bytes\":" << bytes << ",\"gbs_p50\":" << gbs << ",\"raw_ms\":[";
  for (size_t i = 0; i < ms.size(); ++i) j << (i ? "," : "") << ms[i];
  j << "]}" << nl << '}' << '\n';
  std::cout << j.str();

  CUDA_OK(cudaEventDestroy(e0));
  CUDA_OK(cudaEventDestroy(e1));
  cublasDestroy(blas);
  CUDA_OK(cudaStreamDestroy(stream));
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    const Options o = parse(argc, argv);
    if (o.dtype == "fp16") return run<__half>(o);
    if (o.dtype == "bf16") return run<__nv_bfloat16>(o);
    return run<float>(o);
  } catch (const std::exception& e) {
    std::cerr << "gemm_bench: " << e.what() << '\n';
    return 1;
  }
}
