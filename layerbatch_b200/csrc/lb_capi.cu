// C-ABI plumbing: error strings, device info, TMA descriptor encoding, the generic GEMM
// entry point and the device status word.
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "lb_gemm_launch.cuh"
#include "lb_host.h"

namespace lb {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(LB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if (!aligned16(base)) return fail(LB_ERR_INVALID_ARG, "TMA base %p not 16-byte aligned", base);
  for (int i = 0; i < rank - 1; ++i)
    if (strides[i] % 16 != 0)
      return fail(LB_ERR_INVALID_ARG, "TMA stride %llu not a multiple of 16 bytes",
                  (unsigned long long)strides[i]);
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LB_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LB_OK;
}

int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                      uint64_t row_pitch_elems, uint32_t box_rows, uint32_t box_cols) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  return encode(m, base, 2, dims, strides, box);
}

int make_tmap_bf16_3d(CUtensorMap* m, const void* base, uint64_t depth, uint64_t rows,
                      uint64_t cols, uint64_t row_pitch_elems, uint64_t depth_pitch_elems,
                      uint32_t box_rows, uint32_t box_cols) {
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {row_pitch_elems * 2, depth_pitch_elems * 2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  return encode(m, base, 3, dims, strides, box);
}

int make_tmap_bf16_3d_box(CUtensorMap* m, const void* base, uint64_t d2, uint64_t d1,
                          uint64_t d0, uint64_t s2_elems, uint64_t s1_elems, uint32_t b2,
                          uint32_t b1, uint32_t b0) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_elems * 2, s2_elems * 2};
  cuuint32_t box[3] = {b0, b1, b2};
  return encode(m, base, 3, dims, strides, box);
}

static std::atomic<unsigned long long> g_launches{0};

int launched(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(LB_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
  return LB_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LB_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

void record_event(void* ev, cudaStream_t st) {
  if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev), st);
}

int ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<const void*, int>, int>> done;  // ((func, dev), bytes)
  int dev = 0;
  LB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : done)
    if (e.first.first == func && e.first.second == dev) {
      if (e.second >= bytes) return LB_OK;
      LB_CUDA_CHECK(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
      e.second = bytes;
      return LB_OK;
    }
  LB_CUDA_CHECK(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.push_back({{func, dev}, bytes});
  return LB_OK;
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int max_smem_optin() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return n > 0 ? n : 232448;
}


// 256 x 256 tiles of the CTA-pair GEMM for an M x N product.
static long long pair_tiles(long long M, long long N) {
  return ((M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * (N / PAIR_BN);
}

// Whether the CTA-pair GEMM beats the single-CTA one of tile width `bn`: a wave's time
// taken as proportional to the rows each SM loads per k-block (128 + 128 for a pair,
// 128 + bn alone), times the waves of tiles over the SMs.  The q/k/v projection (M 4608,
// N 9216) and o_proj (N 2048) go to pairs; the router logits (N 512: 36 pair tiles for 74
// SM pairs) stay on 128-wide single tiles.
static bool pair_gemm_pays(long long M, long long N, int bn) {
  if (N % PAIR_BN != 0 || M <= 0) return false;
  const long long sms = num_sms();
  const long long waves2 = (pair_tiles(M, N) + sms / 2 - 1) / (sms / 2);
  const long long tiles1 = ((M + GEMM_BM - 1) / GEMM_BM) * (N / bn);
  const long long waves1 = (tiles1 + sms - 1) / sms;
  return waves2 * (GEMM_BM + PAIR_BN / 2) < waves1 * (GEMM_BM + bn);
}

// The dense GEMM behind lb_gemm_bf16 and the library's own projections: checks, tile
// width choice, tensor maps and the launch of the epilogue `epi` (EPI_BF16, EPI_F32_RED or
// EPI_F32_SPLIT; the last writes split ks into out32 + ks * M * ldc).
int gemm_run(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
             int64_t M, int64_t N, int64_t K, int epi, int splits, int* status, cudaStream_t st) {
  LB_REQUIRE(A && B && C, "lb_gemm_bf16: null pointer");
  LB_REQUIRE(M >= 0 && N > 0 && K > 0, "lb_gemm_bf16: bad shape M=%lld N=%lld K=%lld",
             (long long)M, (long long)N, (long long)K);
  LB_REQUIRE(K % 64 == 0, "lb_gemm_bf16: K=%lld must be a multiple of 64", (long long)K);
  LB_REQUIRE(N % 32 == 0, "lb_gemm_bf16: N=%lld must be a multiple of 32", (long long)N);
  LB_REQUIRE(lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0 && lda >= K && ldb >= K && ldc >= N,
             "lb_gemm_bf16: leading dimensions must be >= the row length and multiples of 8");
  LB_REQUIRE(aligned16(A) && aligned16(B) && aligned16(C), "lb_gemm_bf16: unaligned pointer");
  LB_REQUIRE(M <= (1ll << 30) && N <= (1ll << 30), "lb_gemm_bf16: shape too large");
  if (splits < 1) splits = 1;
  LB_REQUIRE(epi != EPI_BF16 || splits == 1, "lb_gemm_bf16: split-K needs an fp32 accumulator");
  LB_REQUIRE((K / 64) % splits == 0, "lb_gemm_bf16: K/64 must divide by splits");
  if (M == 0) return LB_OK;

  int BN = N % 128 == 0 ? 128 : (N % 64 == 0 ? 64 : 32);
  if (N % 256 == 0 && M > 512) {
    // 256-wide tiles unless 128-wide ones finish sooner: a tile's time taken as
    // proportional to the rows it loads (128 of A + BN of B), times the waves of tiles
    // over the SMs (the router logits, M 4608 x N 512: 72 tiles of 256 leave half the
    // SMs idle, 144 tiles of 128 fill them in one wave)
    const long long mt = (M + GEMM_BM - 1) / GEMM_BM;
    auto cost = [&](int bn) {
      const long long tiles = mt * (N / bn) * splits;
      return ((tiles + num_sms() - 1) / num_sms()) * (GEMM_BM + bn);
    };
    BN = cost(256) <= cost(128) ? 256 : 128;
  }
  CUtensorMap tA, tB;
  int rc = make_tmap_bf16_2d(&tA, A, M, K, lda, GEMM_BM, 64);
  if (rc) return rc;
  if (epi == EPI_BF16 && pair_gemm_pays(M, N, BN)) {
    // CTA pairs: 256 x 256 tiles, each CTA loading 128 rows of A and 128 of B
    if ((rc = make_tmap_bf16_2d(&tB, B, N, K, ldb, PAIR_BN / 2, 64))) return rc;
    GemmArgs a = gemm_args_default(status);
    a.m = (int)M;
    a.n_tiles = (int)(N / PAIR_BN);
    a.k_blocks = (int)(K / 64);
    a.out = C;
    a.ldo = ldc;
    a.out_rows = (int)M;
    a.out_cols = (int)N;
    return launch_gemm_pair<6, EPI_BF16, 4>(tA, tB, a, pair_tiles(M, N), st);
  }
  rc = make_tmap_bf16_3d(&tB, B, 1, N, K, ldb, ldb * N, BN, 64);
  if (rc) return rc;
  GemmArgs a = gemm_args_default(status);
  a.m = (int)M;
  a.n_tiles = (int)(N / BN);
  a.splits = splits;
  a.k_blocks = (int)(K / 64) / splits;
  a.out = C;
  a.ldo = ldc;
  a.out_rows = (int)M;
  a.out_cols = (int)N;
  const long long tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (long long)a.n_tiles * splits;
  const int grid = (int)std::min<long long>(tiles, num_sms());
#define LB_GEMM_CASES(E)                                                          \
  switch (BN) {                                                                   \
    case 256: return launch_gemm<256, 4, E>(tA, tB, a, grid, st);                 \
    case 128: return launch_gemm<128, 6, E>(tA, tB, a, grid, st);                 \
    case 64: return launch_gemm<64, 8, E>(tA, tB, a, grid, st);                   \
    default: return launch_gemm<32, 8, E>(tA, tB, a, grid, st);                   \
  }
  if (epi == EPI_F32_RED) LB_GEMM_CASES(EPI_F32_RED)
  if (epi == EPI_F32_SPLIT) LB_GEMM_CASES(EPI_F32_SPLIT)
  LB_GEMM_CASES(EPI_BF16)
#undef LB_GEMM_CASES
}

}  // namespace lb

using namespace lb;

extern "C" {

const char* lb_get_last_error_string(void) { return g_err; }

int lb_version(void) { return 100; }

unsigned long long lb_kernel_launch_count(void) { return g_launches.load(); }

int lb_device_info(int* n_sms, int* sm_version) {
  int dev = 0;
  LB_CUDA_CHECK(cudaGetDevice(&dev));
  int major = 0, minor = 0, n = 0;
  LB_CUDA_CHECK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  LB_CUDA_CHECK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  LB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (n_sms) *n_sms = n;
  if (sm_version) *sm_version = major * 10 + minor;
  return LB_OK;
}

int lb_read_device_status(const void* workspace, int clear, int* status_out) {
  LB_REQUIRE(workspace != nullptr && status_out != nullptr, "null workspace/status pointer");
  LB_CUDA_CHECK(cudaDeviceSynchronize());
  int v = 0;
  LB_CUDA_CHECK(cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost));
  *status_out = v;
  if (clear && v != 0) LB_CUDA_CHECK(cudaMemset(const_cast<void*>(workspace), 0, sizeof(int)));
  return LB_OK;
}

size_t lb_gemm_workspace_size(void) { return 256; }

int lb_qkv_prologue_gemm(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw,
                         void* qkv_out, int64_t ldo, int64_t K, const LbPrologueArgs* a,
                         void* workspace, void* stream) {
  LB_REQUIRE(a != nullptr && x && w_qkv && qkv_out && workspace, "lb_qkv_prologue_gemm: null pointer");
  if (a->head_dim != PRO_D || a->rotary_dim != PRO_GEMM_ROT)
    return fail(LB_ERR_UNSUPPORTED, "lb_qkv_prologue_gemm: needs head_dim 256 and rotary_dim 64 "
                "(got %lld, %lld): use lb_gemm_bf16 + lb_attn_prologue",
                (long long)a->head_dim, (long long)a->rotary_dim);
  const int64_t M = a->num_tokens, Hq = a->num_q_heads, Hkv = a->num_kv_heads;
  LB_REQUIRE(M >= 0 && M <= (1ll << 30) && Hq > 0 && Hkv > 0 && Hq <= 4096 && Hkv <= 4096,
             "lb_qkv_prologue_gemm: bad token / head counts");
  const int64_t N = (2 * Hq + 2 * Hkv) * PRO_D;
  LB_REQUIRE(K > 0 && K % 64 == 0, "lb_qkv_prologue_gemm: K=%lld must be a multiple of 64", (long long)K);
  LB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldo % 8 == 0 && ldx >= K && ldw >= K && ldo >= N,
             "lb_qkv_prologue_gemm: leading dimensions must cover the rows and be multiples of 8");
  LB_REQUIRE(a->q_norm_w && a->k_norm_w && a->positions && a->slot_mapping && a->cos_sin_cache &&
                 a->k_cache && a->v_cache && a->q_out,
             "lb_qkv_prologue_gemm: null pointer in args");
  LB_REQUIRE(aligned16(x) && aligned16(w_qkv) && aligned16(qkv_out) && aligned16(a->q_out) &&
                 aligned16(a->k_cache) && aligned16(a->v_cache) && aligned16(a->q_norm_w) &&
                 aligned16(a->k_norm_w) && aligned16(a->cos_sin_cache),
             "lb_qkv_prologue_gemm: unaligned pointer");
  LB_REQUIRE(a->q_out_stride_tok % 8 == 0 && a->q_out_stride_head % 8 == 0 &&
                 a->q_out_stride_head >= PRO_D,
             "lb_qkv_prologue_gemm: q_out strides must be multiples of 8 elements");
  LB_REQUIRE(a->max_position > 0 && a->num_slots >= 0, "lb_qkv_prologue_gemm: bad cache sizes");
  if (M == 0) return LB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tA, tB;
  int rc = make_tmap_bf16_2d(&tA, x, M, K, ldx, GEMM_BM, 64);
  if (rc) return rc;
  const bool pair = pair_gemm_pays(M, N, PRO_D);
  rc = pair ? make_tmap_bf16_2d(&tB, w_qkv, N, K, ldw, PAIR_BN / 2, 64)
            : make_tmap_bf16_3d(&tB, w_qkv, 1, N, K, ldw, ldw * N, PRO_D, 64);
  if (rc) return rc;
  GemmArgs g = gemm_args_default(static_cast<int*>(workspace));
  g.m = (int)M;
  g.n_tiles = (int)(N / PRO_D);
  g.k_blocks = (int)(K / 64);
  g.out = qkv_out;
  g.ldo = ldo;
  g.out_rows = (int)M;
  g.out_cols = (int)N;
  g.pro = *a;
  if (pair) return launch_gemm_pair<6, EPI_QKV, 8>(tA, tB, g, pair_tiles(M, N), st);
  const long long tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (long long)g.n_tiles;
  const int grid = (int)std::min<long long>(tiles, num_sms());
  return launch_gemm<PRO_D, 4, EPI_QKV>(tA, tB, g, grid, st);
}

int lb_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                 int64_t M, int64_t N, int64_t K, int c_is_fp32, int splits, void* workspace,
                 void* stream) {
  LB_REQUIRE(A && B && C && workspace, "lb_gemm_bf16: null pointer");
  if (splits < 1) splits = 1;
  LB_REQUIRE(c_is_fp32 || splits == 1, "lb_gemm_bf16: split-K needs an fp32 accumulator");
  return gemm_run(A, lda, B, ldb, C, ldc, M, N, K, c_is_fp32 ? EPI_F32_RED : EPI_BF16, splits,
                  static_cast<int*>(workspace), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
