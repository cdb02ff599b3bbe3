// MoE block on sm_100a: router GEMM -> top-k -> permutation -> grouped SwiGLU GEMM
// (routed experts + shared expert in one persistent launch) -> grouped down GEMM with the
// routing weight fused -> shared-expert down GEMM with the sigmoid gate and the weighted
// combine of the routed rows fused into its epilogue.
//
// Packed row layout used by every stage (G = num_local_experts + 1 groups):
//   rows [0, T)                          group 0: shared expert, token order
//   rows [row_start[g], row_start[g+1])  group g >= 1: local expert g-1, pairs ordered
//                                        slot-major then token (torch.where order of
//                                        nanovllm/models/qwen3_5.py:823-831)
#include <algorithm>
#include <cfloat>
#include <mutex>

#include "lb_gemm_launch.cuh"

#include "lb_host.h"
#include "lb_moe_core.h"

namespace lb {

// pairs per chunk of the chunked permutation (k_perm_chunk_*)
constexpr int PERM_CHUNK = 256;
static int perm_chunks(int T, int k) { return (T * k + PERM_CHUNK - 1) / PERM_CHUNK; }

// ------------------------------------------------------------------------------ top-k
// One warp per token.  Softmax in fp32 over E logits, top-k by (value desc, index asc),
// renormalisation over the selected k (qwen3_5.py:770-773).  Optionally the shared-expert
// gate sigmoid(x . w_sg) (qwen3_5.py:903) in fp32.
//
// Selection: the logits are bf16, so each one gets a 32-bit key whose high half orders
// the bf16 values as unsigned integers (-0 taken as +0, NaN below every number) and whose
// low half is 0xFFFF - e: the largest key is the largest value with the lowest expert
// index, and each of the k rounds is one redux.sync max over the warp's untaken keys.
__device__ __forceinline__ uint32_t topk_key(float v, int e) {
  uint32_t b = __float_as_uint(v) >> 16;          // the bf16 bits (v is a bf16 value)
  if ((b & 0x7FFFu) == 0) b = 0;                  // -0 -> +0
  uint32_t ord;
  if ((b & 0x7FFFu) > 0x7F80u) ord = 0;           // NaN
  else ord = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (ord << 16) | (0xFFFFu - (uint32_t)e);
}

__device__ __forceinline__ float topk_key_value(uint32_t key) {
  const uint32_t ord = key >> 16;
  const uint32_t b = (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
  return __uint_as_float(b << 16);
}

template <int VPL>
__global__ void k_router_topk(const __nv_bfloat16* __restrict__ logits, long long ld, int T,
                              int E, int k, int32_t* __restrict__ ids, float* __restrict__ wf,
                              __nv_bfloat16* __restrict__ wb, const __nv_bfloat16* __restrict__ x,
                              const __nv_bfloat16* __restrict__ wsg, int H,
                              float* __restrict__ sg) {
  pdl_entry();
  const int warps_per_block = blockDim.x / 32;
  const int t = blockIdx.x * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  const __nv_bfloat16* row = logits + (long long)t * ld;
  float v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __bfloat162float(row[e]) : -FLT_MAX;
  }
  // shared-expert gate inputs: the first 8 stripes of x[t] and w_sg in flight with the logits
  constexpr int SG_PRE = 8;
  uint4 xa[SG_PRE], xb[SG_PRE];
  const __nv_bfloat16* xr = sg != nullptr ? x + (long long)t * H : nullptr;
  if (sg != nullptr) {
#pragma unroll
    for (int u = 0; u < SG_PRE; ++u) {
      const int h = lane * 8 + 256 * u;
      if (h < H) {
        xa[u] = *reinterpret_cast<const uint4*>(xr + h);
        xb[u] = *reinterpret_cast<const uint4*>(wsg + h);
      }
    }
  }
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < VPL; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (lane + 32 * i < E) z += expf(v[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);

  uint32_t key[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    key[i] = e < E ? topk_key(v[i], e) : 0u;
  }
  unsigned taken = 0;
  float my_p = 0.f, psum = 0.f;
  int my_id = 0;
  for (int j = 0; j < k; ++j) {
    uint32_t best = 0;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (!((taken >> i) & 1u)) best = max(best, key[i]);
    best = __reduce_max_sync(0xffffffffu, best);
    const int bi = (int)(0xFFFFu - (best & 0xFFFFu));
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    const float p = expf(topk_key_value(best) - m) / z;
    psum += p;
    if (lane == j) {
      my_p = p;
      my_id = bi;
    }
  }
  if (lane < k) {
    const float w = my_p / psum;
    const long long o = (long long)t * k + lane;
    ids[o] = my_id;
    if (wf) wf[o] = w;
    if (wb) wb[o] = __float2bfloat16_rn(w);
  }
  if (sg != nullptr) {
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < SG_PRE; ++u) {
      if (lane * 8 + 256 * u < H) {
        const uint4 a = xa[u], b = xb[u];
        acc += bf16_lo(a.x) * bf16_lo(b.x) + bf16_hi(a.x) * bf16_hi(b.x);
        acc += bf16_lo(a.y) * bf16_lo(b.y) + bf16_hi(a.y) * bf16_hi(b.y);
        acc += bf16_lo(a.z) * bf16_lo(b.z) + bf16_hi(a.z) * bf16_hi(b.z);
        acc += bf16_lo(a.w) * bf16_lo(b.w) + bf16_hi(a.w) * bf16_hi(b.w);
      }
    }
    for (int h = lane * 8 + 256 * SG_PRE; h < H; h += 256) {
      const uint4 a = *reinterpret_cast<const uint4*>(xr + h);
      const uint4 b = *reinterpret_cast<const uint4*>(wsg + h);
      acc += bf16_lo(a.x) * bf16_lo(b.x) + bf16_hi(a.x) * bf16_hi(b.x);
      acc += bf16_lo(a.y) * bf16_lo(b.y) + bf16_hi(a.y) * bf16_hi(b.y);
      acc += bf16_lo(a.z) * bf16_lo(b.z) + bf16_hi(a.z) * bf16_hi(b.z);
      acc += bf16_lo(a.w) * bf16_lo(b.w) + bf16_hi(a.w) * bf16_hi(b.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sg[t] = 1.0f / (1.0f + expf(-acc));
  }
}

// sg[t] = sigmoid(x[t] . w_sg) in fp32, one warp per token (qwen3_5.py:903); used when the
// routing is given and the top-k kernel (which also computes it) does not run.  Without
// w_sg (a shared expert called on its own, qwen3_5.py:916-917) the scale is 1.
__global__ void k_shared_gate(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wsg,
                              int T, int H, float* __restrict__ sg) {
  pdl_entry();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  if (wsg == nullptr) {
    if (lane == 0) sg[t] = 1.0f;
    return;
  }
  const __nv_bfloat16* xr = x + (long long)t * H;
  float acc = 0.f;
#pragma unroll 8
  for (int h = lane * 8; h < H; h += 256) {   // unrolled: a lane's loads all in flight
    const uint4 a = *reinterpret_cast<const uint4*>(xr + h);
    const uint4 b = *reinterpret_cast<const uint4*>(wsg + h);
    acc += bf16_lo(a.x) * bf16_lo(b.x) + bf16_hi(a.x) * bf16_hi(b.x);
    acc += bf16_lo(a.y) * bf16_lo(b.y) + bf16_hi(a.y) * bf16_hi(b.y);
    acc += bf16_lo(a.z) * bf16_lo(b.z) + bf16_hi(a.z) * bf16_hi(b.z);
    acc += bf16_lo(a.w) * bf16_lo(b.w) + bf16_hi(a.w) * bf16_hi(b.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) sg[t] = 1.0f / (1.0f + expf(-acc));
}

// ------------------------------------------------------------------------------ permute
// counts[1+e] += #pairs routed to local expert e (block-local histogram first).
__global__ void k_moe_count(const int32_t* __restrict__ ids, int n, int expert_base, int nl,
                            int* __restrict__ counts) {
  pdl_entry();
  extern __shared__ int hist[];
  for (int i = threadIdx.x; i < nl; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < n; f += gridDim.x * blockDim.x) {
    const int e = ids[f] - expert_base;
    if (e >= 0 && e < nl) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nl; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[1 + i], hist[i]);
}

// Exclusive scans: row_start[g] and mtile_start[g] (128-row tiles) over G groups, with
// group 0 (shared expert) holding T rows.  One block of 1024 threads, G <= 2047.  With
// `iota` it also writes the identity map of the shared-expert rows, iota[i] = i for
// i < iota_n.
__global__ void k_moe_scan(const int* __restrict__ counts, int G, int T,
                           int* __restrict__ row_start, int* __restrict__ mtile_start,
                           int32_t* __restrict__ iota, int iota_n) {
  pdl_entry();
  __shared__ int s_rows[1024], s_tiles[1024];
  const int tid = threadIdx.x;
  int r[2], tl[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int g = 2 * tid + i;
    int c = 0;
    if (g < G) c = (g == 0) ? T : counts[g];
    r[i] = c;
    tl[i] = (c + GEMM_BM - 1) / GEMM_BM;
  }
  s_rows[tid] = r[0] + r[1];
  s_tiles[tid] = tl[0] + tl[1];
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    int a = 0, b = 0;
    if (tid >= off) {
      a = s_rows[tid - off];
      b = s_tiles[tid - off];
    }
    __syncthreads();
    s_rows[tid] += a;
    s_tiles[tid] += b;
    __syncthreads();
  }
  const int ex_r = tid ? s_rows[tid - 1] : 0;
  const int ex_t = tid ? s_tiles[tid - 1] : 0;
  if (2 * tid <= G) {
    row_start[2 * tid] = ex_r;
    mtile_start[2 * tid] = ex_t;
  }
  if (2 * tid + 1 <= G) {
    row_start[2 * tid + 1] = ex_r + r[0];
    mtile_start[2 * tid + 1] = ex_t + tl[0];
  }  if (iota != nullptr)
    for (int i = tid; i < iota_n; i += blockDim.x) iota[i] = i;
}

// One block per local expert: scan all pairs in (slot, token) order and assign packed
// rows with a block-wide ballot prefix, so the order is deterministic.
__global__ void k_moe_scatter(const int32_t* __restrict__ ids, const float* __restrict__ w,
                              int T, int k, int expert_base, const int* __restrict__ row_start,
                              int32_t* __restrict__ perm_token, float* __restrict__ perm_w,
                              int32_t* __restrict__ row_of) {
  pdl_entry();
  __shared__ int warp_cnt[32];
  const int g = blockIdx.x + 1;
  const int e_global = expert_base + blockIdx.x;
  const int base = row_start[g];
  const int cnt = row_start[g + 1] - base;
  if (cnt == 0) return;
  const int n = T * k;
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32, nw = blockDim.x / 32;
  int running = 0;
  for (int f0 = 0; f0 < n; f0 += blockDim.x) {
    const int f = f0 + threadIdx.x;
    int t = 0, j = 0;
    bool match = false;
    if (f < n) {
      j = f / T;
      t = f - j * T;
      match = ids[(long long)t * k + j] == e_global;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, match);
    if (lane == 0) warp_cnt[wid] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int i = 0; i < nw; ++i) {
      const int c = warp_cnt[i];
      if (i < wid) before += c;
      total += c;
    }
    if (match) {
      const int r = base + running + before + __popc(bal & ((1u << lane) - 1u));
      perm_token[r] = t;
      if (perm_w) perm_w[r] = w[(long long)t * k + j];
      row_of[(long long)t * k + j] = r;
    }
    running += total;
    __syncthreads();
  }
}

// Identity map of the shared-expert rows [0, T).
__global__ void k_iota(int32_t* __restrict__ p, int n) {
  pdl_entry();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = i;
}

// a_packed[r] = x[perm_token[r]] for packed rows r in [row_begin, *row_end_ptr): one warp
// per row, 16-byte vectors.
__global__ void k_gather_rows(const __nv_bfloat16* __restrict__ x, int H,
                              const int32_t* __restrict__ perm_token,
                              const int* __restrict__ row_end_ptr, int row_begin,
                              __nv_bfloat16* __restrict__ a_packed) {
  pdl_entry();
  const int row_end = *row_end_ptr;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int vpr = H / 8;
  for (int r = row_begin + blockIdx.x * wpb + (int)(threadIdx.x >> 5); r < row_end;
       r += gridDim.x * wpb) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)perm_token[r] * H);
    uint4* dst = reinterpret_cast<uint4*>(a_packed + (long long)r * H);
#pragma unroll 8
    for (int c = lane; c < vpr; c += 32) dst[c] = src[c];
  }
}

// ------------------------------------------------------------------------------ host
void carve_core(Carve& c, size_t T_sh, size_t T_r, size_t k, size_t H, size_t nl, size_t I,
                MoeWs& w) {
  const size_t rows = T_sh + T_r * k;
  w.chunk_hist = c.take<int>((size_t)perm_chunks((int)T_r, (int)k) * nl);
  w.counts = c.take<int>(nl + 2);
  w.row_start = c.take<int>(nl + 2);
  w.mtile_start = c.take<int>(nl + 2);
  w.perm_token = c.take<int32_t>(rows);
  w.perm_w = c.take<float>(rows);
  w.row_of = c.take<int32_t>(T_r * k);
  w.a_packed = c.take<__nv_bfloat16>(rows * H);
  w.act = c.take<__nv_bfloat16>(rows * I);
  w.yw = c.take<__nv_bfloat16>(rows * H);
}

static size_t carve_moe(const LbMoeArgs& a, void* base, MoeWs& w) {
  const size_t T = a.num_tokens, k = a.top_k, H = a.hidden, E = a.num_experts;
  const size_t nl = a.num_local_experts, I = a.inter;
  Carve c(base, ~size_t(0));
  w.status = c.take<int>(64);
  w.logits = c.take<__nv_bfloat16>(a.routing_given ? 0 : T * E);
  w.ids = c.take<int32_t>(T * k);
  w.wf = c.take<float>(a.routing_given ? 0 : T * k);
  w.wb = c.take<__nv_bfloat16>(T * k);
  carve_core(c, a.no_shared ? 0 : T, T, k, H, nl, I, w);
  return c.off + 256;
}

static int check_moe(const LbMoeArgs* a) {
  LB_REQUIRE(a != nullptr, "lb_moe: null args");
  LB_REQUIRE(a->num_tokens >= 0 && a->num_tokens <= (1 << 20), "lb_moe: num_tokens out of range");
  LB_REQUIRE(a->hidden > 0 && a->hidden % 256 == 0 && a->hidden <= 8192,
             "lb_moe: hidden must be a positive multiple of 256 (<= 8192)");
  LB_REQUIRE(a->num_experts > 0 && a->num_experts <= 1024, "lb_moe: num_experts in [1, 1024]");
  LB_REQUIRE(a->top_k > 0 && a->top_k <= 32 && a->top_k <= a->num_experts,
             "lb_moe: top_k in [1, min(32, E)]");
  LB_REQUIRE(a->inter > 0 && a->inter % 128 == 0, "lb_moe: inter must be a multiple of 128");
  LB_REQUIRE(a->no_shared || a->shared_inter == a->inter,
             "lb_moe: shared_inter must equal inter (fused shared-expert group)");
  LB_REQUIRE(a->num_local_experts >= (a->routing_given ? 0 : 1) &&
                 a->num_local_experts <= a->num_experts && a->expert_base >= 0 &&
                 a->expert_base + a->num_local_experts <= a->num_experts,
             "lb_moe: local expert range outside [0, E)");
  LB_REQUIRE(a->routing_given || a->num_experts % 32 == 0,
             "lb_moe: num_experts must be a multiple of 32");
  LB_REQUIRE(a->x && a->out, "lb_moe: null x/out");
  LB_REQUIRE(a->routing_given ? (a->topk_ids && a->topk_weights_f32) : (a->w_router != nullptr),
             "lb_moe: need w_router, or topk_ids + topk_weights_f32 with routing_given");
  LB_REQUIRE(a->num_local_experts == 0 || (a->w_gate_up && a->w_down), "lb_moe: null expert weights");
  LB_REQUIRE(a->no_shared || (a->w_shared_gate && a->w_shared_up && a->w_shared_down),
             "lb_moe: null shared-expert weights");
  LB_REQUIRE(!a->pair_rows == !a->pair_index, "lb_moe: pair_rows and pair_index go together");
  const void* ptrs[] = {a->x, a->out, a->w_router, a->w_gate_up, a->w_down, a->w_shared_gate,
                        a->w_shared_up, a->w_shared_down, a->w_shared_expert_gate, a->pair_rows};
  for (const void* q : ptrs) LB_REQUIRE(q == nullptr || aligned16(q), "lb_moe: tensors must be 16-byte aligned");
  return LB_OK;
}

int launch_topk(const __nv_bfloat16* logits, long long ld, int T, int E, int k, int32_t* ids,
                float* wf, __nv_bfloat16* wb, const __nv_bfloat16* x, const __nv_bfloat16* wsg,
                int H, float* sg, cudaStream_t st) {
  if (T == 0) return LB_OK;
  const int threads = 256, wpb = threads / 32;
  const int grid = (T + wpb - 1) / wpb;
  const int vpl = (E + 31) / 32;
#define LB_TOPK_CASE(V)                                                                   \
  if (vpl <= V) {                                                                         \
    launch_k(k_router_topk<V>, grid, threads, 0, st, logits, ld, T, E, k, ids, wf, wb, x, wsg, H, \
                                               sg);                                       \
    { int _rc = launched("k_router_topk"); if (_rc) return _rc; }                                          \
    return LB_OK;                                                                         \
  }
  LB_TOPK_CASE(2)
  LB_TOPK_CASE(4)
  LB_TOPK_CASE(8)
  LB_TOPK_CASE(16)
  LB_TOPK_CASE(32)
#undef LB_TOPK_CASE
  return fail(LB_ERR_UNSUPPORTED, "router top-k: E=%d too large", E);
}

// Permutation stages shared by lb_moe_permute and lb_moe_forward.
static int run_permute(const int32_t* ids, const float* wf, int T, int k, int expert_base,
                       int nl, int* counts, int* row_start, int* mtile_start, int32_t* perm_token,
                       float* perm_w, int32_t* row_of, cudaStream_t st) {
  const int G = nl + 1;
  const int n = T * k;
  LB_CUDA_CHECK(cudaMemsetAsync(counts, 0, sizeof(int) * (G + 1), st));
  if (n > 0) LB_CUDA_CHECK(cudaMemsetAsync(row_of, 0xff, sizeof(int32_t) * (size_t)n, st));
  if (n > 0) {
    const int grid = std::min(num_sms() * 2, (n + 1023) / 1024);
    launch_k(k_moe_count, std::max(grid, 1), 1024, sizeof(int) * nl, st, ids, n, expert_base, nl, counts);
    { int _rc = launched("k_moe_count"); if (_rc) return _rc; }
  }
  launch_k(k_moe_scan, 1, 1024, 0, st, counts, G, T, row_start, mtile_start, nullptr, 0);
  { int _rc = launched("k_moe_scan"); if (_rc) return _rc; }
  if (T > 0) {
    launch_k(k_iota, std::min(1024, (T + 255) / 256), 256, 0, st, perm_token, T);
    { int _rc = launched("k_iota"); if (_rc) return _rc; }
  }
  if (n > 0) {
    launch_k(k_moe_scatter, nl, 256, 0, st, ids, wf, T, k, expert_base, row_start, perm_token, perm_w,
                                      row_of);
    { int _rc = launched("k_moe_scatter"); if (_rc) return _rc; }
  }
  return LB_OK;
}

// ------------------------------------------------------------------------------ chunked permute
// The (slot, token)-ordered pairs f = j*T + t are cut into chunks of PERM_CHUNK pairs.
// k_perm_chunk_hist counts every local expert per chunk; k_perm_chunk_scan turns the
// counts into each chunk's first packed row per expert (plus row_start / mtile_start);
// k_perm_chunk_scatter walks each chunk in order with one warp and assigns rows, so the
// result equals the sequential definition bit for bit.
__global__ void k_perm_chunk_hist(const int32_t* __restrict__ ids, int T, int k, int expert_base,
                                  int nl, int* __restrict__ chunk_hist,
                                  int32_t* __restrict__ row_of) {
  pdl_entry();
  extern __shared__ int hist[];
  for (int i = threadIdx.x; i < nl; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int n = T * k;
  const int f = blockIdx.x * PERM_CHUNK + threadIdx.x;
  if (threadIdx.x < PERM_CHUNK && f < n) {
    const int j = f / T, t = f - (f / T) * T;
    const int e = ids[(long long)t * k + j] - expert_base;
    if (e >= 0 && e < nl) atomicAdd(&hist[e], 1);
    row_of[(long long)t * k + j] = -1;   // routed nowhere until the scatter assigns a row
  }
  __syncthreads();
  // expert-major layout [nl][n_chunks]: each expert's chunk counts are contiguous
  for (int i = threadIdx.x; i < nl; i += blockDim.x)
    chunk_hist[(long long)i * gridDim.x + blockIdx.x] = hist[i];
}

// One warp per local expert: exclusive prefix of its chunk counts, in place, and the
// expert's total into counts[1 + e].
__global__ void k_perm_expert_scan(int* __restrict__ chunk_hist, int n_chunks, int nl,
                                   int* __restrict__ counts) {
  pdl_entry();
  const int e = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (e >= nl) return;
  int* h = chunk_hist + (long long)e * n_chunks;
  int run = 0;
  for (int c0 = 0; c0 < n_chunks; c0 += 32) {
    const int c = c0 + lane;
    const int v = c < n_chunks ? h[c] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (c < n_chunks) h[c] = run + incl - v;
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) counts[1 + e] = run;
}

// One warp per chunk, pairs in order; equal experts inside a 32-pair step are ranked with
// __match_any_sync, and a per-expert running count in shared memory carries the order
// across steps.
__global__ void k_perm_chunk_scatter(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                     int T, int k, int expert_base, int nl,
                                     const int* __restrict__ chunk_prefix,
                                     const int* __restrict__ row_start,
                                     int32_t* __restrict__ perm_token, float* __restrict__ perm_w,
                                     int32_t* __restrict__ row_of) {
  pdl_entry();
  extern __shared__ int cnt[];
  const int lane = threadIdx.x;
  const int nc = gridDim.x;
  // cnt[e] starts at the first packed row of expert e's pairs in this chunk (unrolled, so
  // that a lane's loads are all in flight before the first shared store)
#pragma unroll 16
  for (int i = lane; i < nl; i += 32)
    cnt[i] = row_start[1 + i] + chunk_prefix[(long long)i * nc + blockIdx.x];
  __syncwarp();
  const int n = T * k;
  const int f0 = blockIdx.x * PERM_CHUNK;
  // the chunk's expert ids, every step's load issued before any is ranked
  constexpr int STEPS = PERM_CHUNK / 32;
  int es[STEPS];
  float ws[STEPS];
#pragma unroll
  for (int u = 0; u < STEPS; ++u) {
    const int f = f0 + 32 * u + lane;
    es[u] = -1;
    ws[u] = 0.f;
    if (f < n) {
      const int j = f / T, t = f - (f / T) * T;
      es[u] = ids[(long long)t * k + j] - expert_base;
      if (perm_w) ws[u] = w[(long long)t * k + j];
    }
  }
#pragma unroll
  for (int u = 0; u < STEPS; ++u) {
    const int f = f0 + 32 * u + lane;
    int e = -1, t = 0, j = 0;
    if (f < n) {
      j = f / T;
      t = f - j * T;
      e = es[u];
      if (e < 0 || e >= nl) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int before = __popc(peers & ((1u << lane) - 1u));
    int r = 0;
    if (e >= 0) r = cnt[e] + before;
    __syncwarp();
    if (e >= 0 && before == 0) cnt[e] += __popc(peers);
    __syncwarp();
    if (e >= 0) {
      perm_token[r] = t;
      if (perm_w) perm_w[r] = ws[u];
      row_of[(long long)t * k + j] = r;
    }
  }
}

// out[t] = bf16( sum over the shared row t and the routed rows row_of[t, :] of yw ),
// one warp per token, fp32 accumulation, 16-byte loads.
template <int MAXS>  // H <= MAXS * 256, H % 256 == 0
__global__ void k_moe_combine(const __nv_bfloat16* __restrict__ yw, const int32_t* __restrict__ row_of,
                              int T, int k, int H, int has_shared,
                              const __nv_bfloat16* __restrict__ pair_rows,
                              const int32_t* __restrict__ pair_index,
                              __nv_bfloat16* __restrict__ out) {
  pdl_entry();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float acc[MAXS][8];
#pragma unroll
  for (int s = 0; s < MAXS; ++s)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[s][i] = 0.f;
  const int stripes = H / 256;
  const int nsrc = pair_index ? 2 * k : k;
  for (int j = has_shared ? -1 : 0; j < nsrc; ++j) {
    const __nv_bfloat16* base;
    if (j < 0) {
      base = yw + (long long)t * H;                       // shared expert row
    } else if (j < k) {
      const int r = row_of[(long long)t * k + j];         // routed row computed here
      if (r < 0) continue;
      base = yw + (long long)r * H;
    } else {
      const int r = pair_index[(long long)t * k + (j - k)];  // routed row computed elsewhere
      if (r < 0) continue;
      base = pair_rows + (long long)r * H;
    }
    const uint4* src = reinterpret_cast<const uint4*>(base) + lane;
    uint4 v[MAXS];
#pragma unroll
    for (int s = 0; s < MAXS; ++s)
      if (s < stripes) v[s] = src[s * 32];
#pragma unroll
    for (int s = 0; s < MAXS; ++s)
      if (s < stripes) {
        acc[s][0] += bf16_lo(v[s].x); acc[s][1] += bf16_hi(v[s].x);
        acc[s][2] += bf16_lo(v[s].y); acc[s][3] += bf16_hi(v[s].y);
        acc[s][4] += bf16_lo(v[s].z); acc[s][5] += bf16_hi(v[s].z);
        acc[s][6] += bf16_lo(v[s].w); acc[s][7] += bf16_hi(v[s].w);
      }
  }
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * H) + lane;
#pragma unroll
  for (int s = 0; s < MAXS; ++s)
    if (s < stripes)
      dst[s * 32] = make_uint4(pack_bf16x2(acc[s][0], acc[s][1]), pack_bf16x2(acc[s][2], acc[s][3]),
                               pack_bf16x2(acc[s][4], acc[s][5]), pack_bf16x2(acc[s][6], acc[s][7]));
}

// Chunked permutation used by lb_moe_permute and lb_moe_forward.  chunk_hist needs
// perm_chunks(T, k) * nl ints of scratch.
static int run_permute_chunked(const int32_t* ids, const float* wf, int T, int k, int expert_base,
                               int nl, int* chunk_hist, int* counts, int* row_start,
                               int* mtile_start, int32_t* perm_token, float* perm_w,
                               int32_t* row_of, cudaStream_t st, int T0) {
  const int n = T * k;
  const int nc = perm_chunks(T, k);
  // k_perm_chunk_hist marks every pair as routed nowhere (row_of = -1) before the scatter
  // fills in the local ones; without it the marking is a memset
  if (n > 0 && !(nc > 0 && nl > 0))
    LB_CUDA_CHECK(cudaMemsetAsync(row_of, 0xff, sizeof(int32_t) * (size_t)n, st));
  if (nc > 0 && nl > 0) {
    launch_k(k_perm_chunk_hist, nc, PERM_CHUNK, sizeof(int) * nl, st, ids, T, k, expert_base, nl, chunk_hist,
             row_of);
    { int _rc = launched("k_perm_chunk_hist"); if (_rc) return _rc; }
    launch_k(k_perm_expert_scan, (nl + 7) / 8, 256, 0, st, chunk_hist, nc, nl, counts);
    { int _rc = launched("k_perm_expert_scan"); if (_rc) return _rc; }
  } else if (nl > 0) {
    LB_CUDA_CHECK(cudaMemsetAsync(counts, 0, sizeof(int) * (nl + 2), st));
  }
  launch_k(k_moe_scan, 1, 1024, 0, st, counts, nl + 1, T0, row_start, mtile_start,
           T0 > 0 ? perm_token : nullptr, T0);
  { int _rc = launched("k_moe_scan"); if (_rc) return _rc; }
  if (nc > 0 && nl > 0) {
    launch_k(k_perm_chunk_scatter, nc, 32, sizeof(int) * nl, st, ids, wf, T, k, expert_base, nl, chunk_hist,
                                                           row_start, perm_token, perm_w, row_of);
    { int _rc = launched("k_perm_chunk_scatter"); if (_rc) return _rc; }
  }
  return LB_OK;
}

// ------------------------------------------------------------------------------ core
int moe_core(const MoeCore& c, const MoeWs& w, cudaStream_t st) {
  const int T = c.T_r, H = c.H, k = c.k, I = c.I, nl = c.nl;
  const int T0 = c.T_sh;
  const int G = nl + 1;
  const bool shared = T0 > 0;
  const int32_t* ids = c.ids;
  const float* wf = c.wf;
  // 3. permutation (routed pairs of the local experts) and gather of their input rows
  int rc = run_permute_chunked(ids, wf, T, k, c.expert_base, nl, w.chunk_hist, w.counts,
                               w.row_start, w.mtile_start, w.perm_token, w.perm_w, w.row_of, st,
                               T0);
  if (rc) return rc;
  if (nl > 0) {
    const long long rows_r = (long long)T * k;
    const int grid = (int)std::max<long long>(1, std::min<long long>(num_sms() * 8, (rows_r + 7) / 8));
    launch_k(k_gather_rows, grid, 256, 0, st, c.x_r, H, w.perm_token, w.row_start + G, T0, w.a_packed);
    { int _rc = launched("k_gather_rows"); if (_rc) return _rc; }
  }
  const long long rows = (long long)T0 + (long long)T * k;
  // token tiles over all groups <= rows / TN + groups
  auto max_units = [&](int TN, int n_fb) {
    return (long long)n_fb * (rows / TN + G);
  };
  const bool any_gemm = shared || nl > 0;

  // 4. grouped gate/up GEMM with SwiGLU: act[rows, I].  Accumulator 0 holds gate rows
  //    fb*128.., accumulator 1 the up rows I + fb*128.. of the same expert.
  if (any_gemm) {
    // 128-token tiles, double-buffered accumulators, 4-stage ring (48 KB per stage); two
    // epilogue warps per TMEM lane quadrant for the SwiGLU epilogue
    constexpr int TN = 128, NBUF = 2, STAGES = 4, EPW = 8;
    CUtensorMap tX, tXsh, tW, tW0, tW1;
    if ((rc = make_tmap_bf16_2d(&tX, w.a_packed, rows, H, H, TOK_BOX, 64))) return rc;
    if ((rc = make_tmap_bf16_2d(&tXsh, shared ? c.x_sh : c.x_r, shared ? T0 : T, H, H, TOK_BOX, 64)))
      return rc;
    if (nl > 0 && (rc = make_tmap_bf16_3d(&tW, c.w_gate_up, nl, 2 * I, H, H, (uint64_t)2 * I * H,
                                          TOK_FB, 64)))
      return rc;
    if (shared) {
      if ((rc = make_tmap_bf16_3d(&tW0, c.w_sh_gate, 1, I, H, H, (uint64_t)I * H, TOK_FB, 64)))
        return rc;
      if ((rc = make_tmap_bf16_3d(&tW1, c.w_sh_up, 1, I, H, H, (uint64_t)I * H, TOK_FB, 64)))
        return rc;
    }
    if (nl == 0) tW = tW0;
    if (!shared) tW0 = tW1 = tW;
    TokArgs g{};
    g.status = w.status;
    g.row_start = w.row_start;
    g.num_groups = G;
    g.n_fb = I / TOK_FB;
    g.fb_stride = TOK_FB;
    g.acc1_off = I;
    g.acc1_off_sh = 0;
    g.k_blocks = H / 64;
    g.shared_group = shared ? 0 : -1;
    g.w_group_base = 1;
    g.out = w.act;
    g.ldo = I;
    g.out_rows = (int)rows;
    g.out_cols = I;
    const int grid = (int)std::min<long long>(num_sms(), max_units(TN, g.n_fb));
    record_event(c.events ? c.events[0] : nullptr, st);
    if ((rc = launch_gemm_tok<TN, NBUF, STAGES, TOK_EPI_SWIGLU, EPW>(tW, tW0, tW1, tX, tXsh, g, grid, st)))
      return rc;
    record_event(c.events ? c.events[1] : nullptr, st);
  }
  // 5. grouped down GEMM of every group (shared expert = group 0), each row scaled by its
  //    routing weight (shared rows: sigmoid gate): yw[rows, H].  Accumulators 0 / 1 hold
  //    output features fb*256 + [0, 128) / [128, 256).
  if (any_gemm) {
    constexpr int TN = 128, NBUF = 2, STAGES = 4, EPW = 8;
    CUtensorMap tX, tW, tWs;
    if ((rc = make_tmap_bf16_2d(&tX, w.act, rows, I, I, TOK_BOX, 64))) return rc;
    if (nl > 0 && (rc = make_tmap_bf16_3d(&tW, c.w_down, nl, H, I, I, (uint64_t)H * I, TOK_FB, 64)))
      return rc;
    if (shared && (rc = make_tmap_bf16_3d(&tWs, c.w_sh_down, 1, H, I, I, (uint64_t)H * I, TOK_FB, 64)))
      return rc;
    if (nl == 0) tW = tWs;
    if (!shared) tWs = tW;
    TokArgs g{};
    g.status = w.status;
    g.row_start = w.row_start;
    g.num_groups = G;
    g.n_fb = H / (2 * TOK_FB);
    g.fb_stride = 2 * TOK_FB;
    g.acc1_off = TOK_FB;
    g.acc1_off_sh = TOK_FB;
    g.k_blocks = I / 64;
    g.shared_group = shared ? 0 : -1;
    g.w_group_base = 1;
    g.row_scale = w.perm_w;
    g.out = w.yw;
    g.ldo = H;
    g.out_rows = (int)rows;
    g.out_cols = H;
    const int grid = (int)std::min<long long>(num_sms(), max_units(TN, g.n_fb));
    record_event(c.events ? c.events[2] : nullptr, st);
    if ((rc = launch_gemm_tok<TN, NBUF, STAGES, TOK_EPI_SCALE, EPW>(tW, tWs, tWs, tX, tX, g, grid, st)))
      return rc;
    record_event(c.events ? c.events[3] : nullptr, st);
  }
  return LB_OK;
}

// ------------------------------------------------------------------------------ no-alloc
// Fixed scratch for lb_moe_permute_noalloc, for callers that may not allocate device
// memory.  It lives in this module's static device memory: every GPU that loads the
// library holds LB_NOALLOC_SCRATCH_INTS * 4 bytes (8,464 bytes) of it until the process
// exits, and every call on a device shares it.
constexpr int LB_NOALLOC_MAX_LOCAL_EXPERTS = 1024;
// k_moe_scatter runs one CTA per local expert over all T*k pairs: the cap bounds a call's
// work to num_local_experts * 2^20 id reads (L2-resident).
constexpr long long LB_NOALLOC_MAX_PAIRS = 1ll << 20;
constexpr int LB_NOALLOC_SCRATCH_INTS = 64 + 2 * (LB_NOALLOC_MAX_LOCAL_EXPERTS + 2);
static __device__ __align__(256) int g_permute_scratch[LB_NOALLOC_SCRATCH_INTS];

constexpr int LB_NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static int* g_noalloc_addr[LB_NOALLOC_MAX_DEVICES] = {};

// Device address of g_permute_scratch on the current device.  In host code the array's
// name only stands in for the symbol; the address a kernel may use comes from
// cudaGetSymbolAddress, looked up once per device (with that device current) and cached
// for the life of the process (a cudaDeviceReset invalidates it).
static int noalloc_scratch(int** out) {
  int dev = -1;
  LB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= LB_NOALLOC_MAX_DEVICES)
    return fail(LB_ERR_UNSUPPORTED, "lb_moe_permute_noalloc: device %d beyond the %d cached",
                dev, LB_NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(LB_ERR_CUDA, "lb_moe_permute_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_noalloc_addr[dev] = static_cast<int*>(p);
  }
  *out = g_noalloc_addr[dev];
  return LB_OK;
}

}  // namespace lb

using namespace lb;

extern "C" {

int lb_router_topk(const void* logits, int64_t ld, int64_t T, int64_t E, int64_t k, int32_t* ids,
                   float* weights_f32, void* weights_bf16, void* stream) {
  LB_REQUIRE(logits && ids, "lb_router_topk: null pointer");
  LB_REQUIRE(T >= 0 && E > 0 && E <= 1024 && k > 0 && k <= 32 && k <= E && ld >= E,
             "lb_router_topk: need 0<k<=min(32,E), E<=1024, ld>=E");
  return launch_topk(static_cast<const __nv_bfloat16*>(logits), ld, (int)T, (int)E, (int)k, ids,
                     weights_f32, static_cast<__nv_bfloat16*>(weights_bf16), nullptr, nullptr, 0,
                     nullptr, static_cast<cudaStream_t>(stream));
}

size_t lb_moe_permute_workspace_size(int64_t T, int64_t k, int64_t nl) {
  const size_t nc = (size_t)((T * k + PERM_CHUNK - 1) / PERM_CHUNK);
  return 256 + 4 * 256 + 2 * sizeof(int) * (size_t)(nl + 2) + sizeof(int) * nc * (size_t)nl;
}

int lb_moe_permute(const int32_t* ids, int64_t T, int64_t k, int64_t expert_base,
                   int64_t nl, int32_t* row_start, int32_t* perm_token, int32_t* row_of,
                   void* workspace, size_t workspace_bytes, void* stream) {
  LB_REQUIRE(row_start && (T == 0 || (ids && perm_token && row_of)),
             "lb_moe_permute: null pointer");
  LB_REQUIRE(T >= 0 && k > 0 && k <= 32 && nl > 0 && nl <= 2046 && expert_base >= 0,
             "lb_moe_permute: bad sizes");
  LB_REQUIRE(T * k < (1ll << 30), "lb_moe_permute: too many pairs");
  if (!workspace || workspace_bytes < lb_moe_permute_workspace_size(T, k, nl))
    return fail(LB_ERR_WORKSPACE, "lb_moe_permute: workspace too small");
  Carve c(workspace, workspace_bytes);
  c.take<int>(64);  // status word
  int* mt = c.take<int>(nl + 2);
  int* counts = c.take<int>(nl + 2);
  int* chunk_hist = c.take<int>((size_t)perm_chunks((int)T, (int)k) * nl);
  return run_permute_chunked(ids, nullptr, (int)T, (int)k, (int)expert_base, (int)nl, chunk_hist,
                             counts, row_start, mt, perm_token, nullptr, row_of,
                             static_cast<cudaStream_t>(stream), (int)T);
}

int lb_moe_permute_noalloc(const int32_t* ids, int64_t T, int64_t k, int64_t expert_base,
                           int64_t nl, int32_t* row_start, int32_t* perm_token, int32_t* row_of,
                           void* stream) {
  LB_REQUIRE(row_start && (T == 0 || (ids && perm_token && row_of)),
             "lb_moe_permute_noalloc: null pointer");
  LB_REQUIRE(T >= 0 && k > 0 && k <= 32 && expert_base >= 0 && nl > 0,
             "lb_moe_permute_noalloc: bad sizes");
  if (T * k > LB_NOALLOC_MAX_PAIRS)
    return fail(LB_ERR_UNSUPPORTED,
                "lb_moe_permute_noalloc: %lld (token, slot) pairs exceed the limit of %lld "
                "(use lb_moe_permute with a workspace)",
                (long long)(T * k), LB_NOALLOC_MAX_PAIRS);
  if (nl > LB_NOALLOC_MAX_LOCAL_EXPERTS)
    return fail(LB_ERR_UNSUPPORTED,
                "lb_moe_permute_noalloc: %lld local experts exceed the fixed scratch limit of %d "
                "(use lb_moe_permute with a workspace)",
                (long long)nl, LB_NOALLOC_MAX_LOCAL_EXPERTS);
  int* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // layout: [status x64][counts: nl+2][mtile_start: nl+2]; run_permute zeroes the counts
  // (and presets row_of) on the stream before use, so a previous call's contents are harmless
  int* counts = scratch + 64;
  int* mt = counts + (nl + 2);
  return run_permute(ids, nullptr, (int)T, (int)k, (int)expert_base, (int)nl, counts, row_start,
                     mt, perm_token, nullptr, row_of, static_cast<cudaStream_t>(stream));
}

int lb_moe_workspace_size(const LbMoeArgs* a, size_t* bytes) {
  int rc = check_moe(a);
  if (rc) return rc;
  LB_REQUIRE(bytes != nullptr, "lb_moe_workspace_size: null output");
  MoeWs w;
  *bytes = carve_moe(*a, nullptr, w);
  return LB_OK;
}

int lb_moe_forward(const LbMoeArgs* a, void* stream) {
  int rc = check_moe(a);
  if (rc) return rc;
  MoeWs w;
  const size_t need = carve_moe(*a, a->workspace, w);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(LB_ERR_WORKSPACE, "lb_moe_forward: workspace %zu < %zu bytes",
                (size_t)a->workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = (int)a->num_tokens, H = (int)a->hidden, E = (int)a->num_experts;
  const int k = (int)a->top_k, I = (int)a->inter, nl = (int)a->num_local_experts;
  const bool shared = !a->no_shared;
  const int T0 = shared ? T : 0;  // rows of group 0 (the shared expert)
  if (T == 0) return LB_OK;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a->x);
  const int32_t* ids;
  const float* wf;
  if (a->routing_given) {
    ids = a->topk_ids;
    wf = a->topk_weights_f32;
    if (shared) {
      // the shared-expert gate lands in perm_w[0:T) (see below)
      launch_k(k_shared_gate, (T * 32 + 255) / 256, 256, 0, st, 
          x, static_cast<const __nv_bfloat16*>(a->w_shared_expert_gate), T, H, w.perm_w);
      { int _rc = launched("k_shared_gate"); if (_rc) return _rc; }
    }
  } else {
    __nv_bfloat16* logits =
        a->router_logits ? static_cast<__nv_bfloat16*>(a->router_logits) : w.logits;
    int32_t* ids_out = a->topk_ids ? a->topk_ids : w.ids;
    __nv_bfloat16* wb = a->topk_weights ? static_cast<__nv_bfloat16*>(a->topk_weights) : w.wb;
    // 1. router logits [T, E] = x . W_router^T (bf16 out, fp32 accumulate)
    rc = lb_gemm_bf16(a->x, H, a->w_router, H, logits, E, T, E, H, 0, 1, w.status, stream);
    if (rc) return rc;
    // 2. top-k + shared-expert gate.  The gate lands in perm_w[0:T): rows [0,T) of every
    //    packed buffer are the shared expert's, so the down GEMM scales them by it exactly
    //    as it scales routed rows by their routing weight.
    const bool gated = shared && a->w_shared_expert_gate != nullptr;
    rc = launch_topk(logits, E, T, E, k, ids_out, w.wf, wb, x,
                     static_cast<const __nv_bfloat16*>(a->w_shared_expert_gate), H,
                     gated ? w.perm_w : nullptr, st);
    if (rc) return rc;
    if (shared && !gated) {   // an ungated shared expert: scale 1
      launch_k(k_shared_gate, (T * 32 + 255) / 256, 256, 0, st, x,
               static_cast<const __nv_bfloat16*>(nullptr), T, H, w.perm_w);
      { int _rc = launched("k_shared_gate"); if (_rc) return _rc; }
    }
    ids = ids_out;
    wf = w.wf;
  }
  // 3.-5. permutation, gather, grouped gate/up (SwiGLU) and down GEMMs
  {
    MoeCore c{};
    c.T_sh = T0;
    c.T_r = T;
    c.H = H;
    c.k = k;
    c.I = I;
    c.nl = nl;
    c.expert_base = (int)a->expert_base;
    c.x_sh = x;
    c.x_r = x;
    c.ids = ids;
    c.wf = wf;
    c.w_gate_up = a->w_gate_up;
    c.w_down = a->w_down;
    c.w_sh_gate = a->w_shared_gate;
    c.w_sh_up = a->w_shared_up;
    c.w_sh_down = a->w_shared_down;
    c.events = a->timing_events;
    if ((rc = moe_core(c, w, st))) return rc;
  }
  // 6. combine: out[t] = yw[t] (shared) + sum_j yw[row_of[t, j]] + sum_j pair_rows[pair_index[t, j]]
  {
    const int blocks = (T * 32 + 255) / 256;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a->out);
    const __nv_bfloat16* pr = static_cast<const __nv_bfloat16*>(a->pair_rows);
    if (H <= 2048)
      launch_k(k_moe_combine<8>, blocks, 256, 0, st, w.yw, w.row_of, T, k, H, shared, pr, a->pair_index, out);
    else if (H <= 4096)
      launch_k(k_moe_combine<16>, blocks, 256, 0, st, w.yw, w.row_of, T, k, H, shared, pr, a->pair_index, out);
    else
      launch_k(k_moe_combine<32>, blocks, 256, 0, st, w.yw, w.row_of, T, k, H, shared, pr, a->pair_index, out);
    { int _rc = launched("k_moe_combine"); if (_rc) return _rc; }
  }
  (void)E;
  return LB_OK;
}

}  // extern "C"
