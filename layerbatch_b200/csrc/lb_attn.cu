// Paged attention hot path: KV-cache store, POD attention (prefill + decode in one
// persistent launch), split merge with the sigmoid output gate, and the o_proj GEMM.
#include <algorithm>

#include "lb_gemm_launch.cuh"
#include "lb_host.h"
#include "lb_pod.cuh"
#include "lb_prologue.cuh"

namespace lb {

// One warp per token row: copy k/v rows of `row_elems` bf16 into the slot given by
// slot_mapping (skip -1; out-of-range slots are skipped too).
__global__ void k_store_kvcache(const __nv_bfloat16* __restrict__ k, long long ks,
                                const __nv_bfloat16* __restrict__ v, long long vs,
                                __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                const int32_t* __restrict__ slots, int n, long long num_slots,
                                int row_elems) {
  pdl_entry();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (w >= n) return;
  const long long s = slots[w];
  if (s < 0 || s >= num_slots) return;
  const uint4* ksrc = reinterpret_cast<const uint4*>(k + (long long)w * ks);
  const uint4* vsrc = reinterpret_cast<const uint4*>(v + (long long)w * vs);
  uint4* kdst = reinterpret_cast<uint4*>(kc + s * row_elems);
  uint4* vdst = reinterpret_cast<uint4*>(vc + s * row_elems);
  for (int i = lane; i < row_elems / 8; i += 32) {
    kdst[i] = ksrc[i];
    vdst[i] = vsrc[i];
  }
}


// ------------------------------------------------------------------------------ prologue
// The standalone prologue (lb_attn_prologue): one block per task of PRO_TASK_TOKENS
// tokens (grid-stride), 8 warps on its rows (lb_prologue.cuh).
__global__ void __launch_bounds__(256) k_attn_prologue(const LbPrologueArgs a) {
  pdl_entry();
  __shared__ ProStage st;
  const int tasks = (int)((a.num_tokens + PRO_TASK_TOKENS - 1) / PRO_TASK_TOKENS);
  for (int t = blockIdx.x; t < tasks; t += gridDim.x) {
    const int tok0 = t * PRO_TASK_TOKENS;
    const int ntok = (int)(a.num_tokens - tok0) < PRO_TASK_TOKENS ? (int)(a.num_tokens - tok0)
                                                                    : PRO_TASK_TOKENS;
    prologue_task(a, nullptr, tok0, ntok, &st, threadIdx.x / 32, 8, threadIdx.x % 32, a.status);
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------ plan
// One block.  Phase 1: per-sequence item counts and block-wide exclusive scans give every
// sequence its first item slots (kept in shared memory).  Phase 2: each thread writes the
// decode items of its own sequences; prefill sequences (many items each) are written by
// the lanes of their thread's warp together.  Queue order is longest first, so the
// dynamic scheduler ends on short items: prefill tiles latest query tile first; decode
// items all full-length splits first, then every sequence's shorter last split.
__global__ void k_pod_plan(const int32_t* __restrict__ ctx_lens, const int32_t* __restrict__ cu,
                           int B, int Hq, int Hkv, int split_tokens, int max_splits,
                           int max_ctx, int pf_cap, int dec_cap, int4* __restrict__ pf_items,
                           int* __restrict__ counters, int4* __restrict__ dec_items,
                           int* __restrict__ seq_ready, int* __restrict__ status) {
  pdl_entry();
  __shared__ int s_pf[1024], s_full[1024], s_rem[1024];
  extern __shared__ int s_off[];  // [3 * B]: first prefill / full-split / last-split item
  const int tid = threadIdx.x;
  const int per = (B + 1023) / 1024;
  const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
  int npf = 0, nfull = 0, nrem = 0;
  for (int b = b0; b < b1; ++b) {
    const int qlen = cu[b + 1] - cu[b];
    const int ctx = ctx_lens[b];
    if (qlen <= 0 || ctx < qlen || ctx > max_ctx) {
      if (qlen != 0) report(status, LB_DEV_BAD_INDEX);
      continue;
    }
    if (qlen == 1) {
      nfull += Hkv * (ctx / split_tokens);
      nrem += (ctx % split_tokens) ? Hkv : 0;
    } else {
      npf += Hq * ((qlen + POD_KV - 1) / POD_KV);
    }
  }
  // inclusive block scans of the three counts: within each warp by shuffles, then the
  // 32 warp totals by one warp (two block barriers instead of one pair per step)
  {
    const int lane = tid & 31, wid = tid >> 5;
    int a = npf, c = nfull, d = nrem;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int xa = __shfl_up_sync(0xffffffffu, a, o);
      const int xc = __shfl_up_sync(0xffffffffu, c, o);
      const int xd = __shfl_up_sync(0xffffffffu, d, o);
      if (lane >= o) {
        a += xa;
        c += xc;
        d += xd;
      }
    }
    if (lane == 31) {
      s_pf[wid] = a;
      s_full[wid] = c;
      s_rem[wid] = d;
    }
    __syncthreads();
    if (wid == 0) {
      int wa = s_pf[lane], wc = s_full[lane], wd = s_rem[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int xa = __shfl_up_sync(0xffffffffu, wa, o);
        const int xc = __shfl_up_sync(0xffffffffu, wc, o);
        const int xd = __shfl_up_sync(0xffffffffu, wd, o);
        if (lane >= o) {
          wa += xa;
          wc += xc;
          wd += xd;
        }
      }
      s_pf[32 + lane] = wa;   // inclusive prefix of the warp totals
      s_full[32 + lane] = wc;
      s_rem[32 + lane] = wd;
    }
    __syncthreads();
    const int pa = wid ? s_pf[32 + wid - 1] : 0;
    const int pc = wid ? s_full[32 + wid - 1] : 0;
    const int pd = wid ? s_rem[32 + wid - 1] : 0;
    __syncthreads();   // every thread has read the warp prefixes before they are overwritten
    s_pf[tid] = a + pa;
    s_full[tid] = c + pc;
    s_rem[tid] = d + pd;
    __syncthreads();
  }
  const int total_full = s_full[1023];
  int opf = s_pf[tid] - npf, ofull = s_full[tid] - nfull, orem = total_full + s_rem[tid] - nrem;
  for (int b = b0; b < b1; ++b) {
    s_off[b] = opf;
    s_off[B + b] = ofull;
    s_off[2 * B + b] = orem;
    const int qlen = cu[b + 1] - cu[b];
    const int ctx = ctx_lens[b];
    if (qlen <= 0 || ctx < qlen || ctx > max_ctx) continue;
    if (qlen == 1) {
      ofull += Hkv * (ctx / split_tokens);
      orem += (ctx % split_tokens) ? Hkv : 0;
    } else {
      opf += Hq * ((qlen + POD_KV - 1) / POD_KV);
    }
  }
  __syncthreads();
  // Phase 2: every thread writes the decode items of its own sequences; the prefill
  // sequences of a warp's threads are written by the whole warp, one after another.
  const int lane = tid % 32;
  for (int kk = 0; kk < per; ++kk) {
    const int b = b0 + kk;
    int qlen = 0, ctx = 0;
    bool valid = b < b1;
    if (valid) {
      qlen = cu[b + 1] - cu[b];
      ctx = ctx_lens[b];
      valid = !(qlen <= 0 || ctx < qlen || ctx > max_ctx);
    }
    if (valid && qlen == 1) {
      const int nf = ctx / split_tokens;
      const int n = Hkv * nf;
      const int o = s_off[B + b];
      for (int i = 0; i < n; ++i)
        if (o + i < dec_cap) dec_items[o + i] = make_int4(b, i % Hkv, i / Hkv, 0);
      if (ctx % split_tokens) {
        const int orr = s_off[2 * B + b];
        for (int i = 0; i < Hkv; ++i)
          if (orr + i < dec_cap) dec_items[orr + i] = make_int4(b, i, nf, 0);
      }
    }
    unsigned pfm = __ballot_sync(0xffffffffu, valid && qlen > 1);
    while (pfm) {
      const int src = __ffs(pfm) - 1;
      pfm &= pfm - 1;
      const int bb = __shfl_sync(0xffffffffu, b, src);
      const int ql = __shfl_sync(0xffffffffu, qlen, src);
      const int nqt = (ql + POD_KV - 1) / POD_KV;
      const int n = Hq * nqt;
      const int o = s_off[bb];
      for (int i = lane; i < n; i += 32)
        if (o + i < pf_cap) pf_items[o + i] = make_int4(bb, i % Hq, nqt - 1 - i / Hq, 0);
    }
  }
  if (tid == 1023) {
    const int tp = s_pf[1023], td = total_full + s_rem[1023];
    if (tp > pf_cap || td > dec_cap) report(status, LB_DEV_BAD_INDEX);
    counters[0] = min(tp, pf_cap);
    counters[1] = 0;
    counters[2] = min(td, dec_cap);
    counters[3] = 0;
    counters[4] = 0;   // fused prologue: next task
    counters[5] = 0;   // fused prologue: tasks finished
  }
  // fused prologue: no new token of any sequence is stored yet
  if (seq_ready)
    for (int b = tid; b < B; b += 1024) seq_ready[b] = 0;
}

// ------------------------------------------------------------------------------ merge
// Decode sequences: combine the split partials by their log2-sum-exp, apply
// sigmoid(gate) and write the bf16 o_proj input row (and optionally the raw output).
// One CTA per (sequence, group of `hpc` heads), 32 threads per head (8 dims each).  The
// partials' loads are issued four splits at a time before any is used, so a CTA waits
// for about one memory latency per four splits, not one per split.  The sums run over
// the splits in order, as before the loads were batched.
constexpr int MERGE_SPLIT_BATCH = 4;
__global__ void k_pod_merge(const int32_t* __restrict__ ctx_lens, const int32_t* __restrict__ cu,
                            int Hq, int hpc, int split_tokens, int max_splits, int max_ctx,
                            const float* __restrict__ part_o, const float* __restrict__ part_lse,
                            const __nv_bfloat16* __restrict__ gate, long long gst, long long gsh,
                            __nv_bfloat16* __restrict__ ogated, __nv_bfloat16* __restrict__ attn_out) {
  pdl_entry();
  extern __shared__ float wts[];  // [max_splits][hpc]
  const int groups = Hq / hpc;
  const int b = blockIdx.x / groups;
  const int h0 = (blockIdx.x - b * groups) * hpc;
  const int q0 = cu[b];
  if (cu[b + 1] - q0 != 1) return;
  const int ctx = ctx_lens[b];
  const int ns = (ctx >= 1 && ctx <= max_ctx) ? min(max_splits, (ctx + split_tokens - 1) / split_tokens) : 0;
  const long long pb = (long long)b * max_splits;
  for (int e = threadIdx.x; e < ns * hpc; e += blockDim.x) {
    const int sp = e / hpc, hl = e - (e / hpc) * hpc;
    wts[sp * hpc + hl] = part_lse[(pb + sp) * Hq + h0 + hl];
  }
  __syncthreads();
  for (int hl = threadIdx.x; hl < hpc; hl += blockDim.x) {
    float m = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) m = fmaxf(m, wts[sp * hpc + hl]);
    float sum = 0.f;
    for (int sp = 0; sp < ns; ++sp) {
      const float w = exp2f(wts[sp * hpc + hl] - m);
      wts[sp * hpc + hl] = w;
      sum += w;
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    for (int sp = 0; sp < ns; ++sp) wts[sp * hpc + hl] *= inv;
  }
  __syncthreads();
  const int HD = Hq * POD_D;
  for (int i = h0 * POD_D + threadIdx.x * 8; i < (h0 + hpc) * POD_D; i += blockDim.x * 8) {
    const int h = i / POD_D, d = i % POD_D, hl = h - h0;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < ns; s0 += MERGE_SPLIT_BATCH) {
      float4 xa[MERGE_SPLIT_BATCH], xb[MERGE_SPLIT_BATCH];
#pragma unroll
      for (int u = 0; u < MERGE_SPLIT_BATCH; ++u) {
        if (s0 + u < ns) {
          const float4* src = reinterpret_cast<const float4*>(part_o + ((pb + s0 + u) * Hq + h) * POD_D + d);
          xa[u] = src[0];
          xb[u] = src[1];
        }
      }
#pragma unroll
      for (int u = 0; u < MERGE_SPLIT_BATCH; ++u) {
        if (s0 + u < ns) {
          const float w = wts[(s0 + u) * hpc + hl];
          const float4 x0 = xa[u], x1 = xb[u];
          o[0] += w * x0.x; o[1] += w * x0.y; o[2] += w * x0.z; o[3] += w * x0.w;
          o[4] += w * x1.x; o[5] += w * x1.y; o[6] += w * x1.z; o[7] += w * x1.w;
        }
      }
    }
    if (ogated) {
      float gv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (gate) {
        const uint4 g = *reinterpret_cast<const uint4*>(gate + (long long)q0 * gst + (long long)h * gsh + d);
        gv[0] = sigmoid_f(bf16_lo(g.x)); gv[1] = sigmoid_f(bf16_hi(g.x));
        gv[2] = sigmoid_f(bf16_lo(g.y)); gv[3] = sigmoid_f(bf16_hi(g.y));
        gv[4] = sigmoid_f(bf16_lo(g.z)); gv[5] = sigmoid_f(bf16_hi(g.z));
        gv[6] = sigmoid_f(bf16_lo(g.w)); gv[7] = sigmoid_f(bf16_hi(g.w));
      }
      uint4 outv;
      outv.x = pack_bf16x2(o[0] * gv[0], o[1] * gv[1]);
      outv.y = pack_bf16x2(o[2] * gv[2], o[3] * gv[3]);
      outv.z = pack_bf16x2(o[4] * gv[4], o[5] * gv[5]);
      outv.w = pack_bf16x2(o[6] * gv[6], o[7] * gv[7]);
      *reinterpret_cast<uint4*>(ogated + (long long)q0 * HD + i) = outv;
    }
    if (attn_out) {
      uint4 r;
      r.x = pack_bf16x2(o[0], o[1]);
      r.y = pack_bf16x2(o[2], o[3]);
      r.z = pack_bf16x2(o[4], o[5]);
      r.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(attn_out + (long long)q0 * HD + i) = r;
    }
  }
}

// out[r, c] = sum over s = 0..splits-1 (in that order) of parts[s][r, c]: the split-K
// partial slices of the o_proj GEMM (EPI_F32_SPLIT) added in a fixed order, so the result
// does not depend on which split finished first; written as bf16 or fp32.
__global__ void k_splitk_reduce(const float* __restrict__ parts, int splits, long long rows,
                                int cols, __nv_bfloat16* __restrict__ out_bf16,
                                float* __restrict__ out_f32, long long ld_out) {
  pdl_entry();
  const long long slice = rows * cols;
  const int groups = cols / 4;   // 4-float groups per row
  // one thread per 4-float group of the output (grid-stride); a thread's slice loads are
  // issued eight at a time before they are added, in split order
  for (long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x; gi < rows * groups;
       gi += (long long)gridDim.x * blockDim.x) {
    const long long r = gi / groups;
    const int c = (int)(gi - r * groups) * 4;
    const float* src = parts + r * cols + c;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int s0 = 1; s0 < splits; s0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < splits) v[u] = *reinterpret_cast<const float4*>(src + (s0 + u) * slice);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + u < splits) {
          acc.x += v[u].x;
          acc.y += v[u].y;
          acc.z += v[u].z;
          acc.w += v[u].w;
        }
      }
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(out_f32 + r * ld_out + c) = acc;
    } else {
      uint2 o;
      o.x = pack_bf16x2(acc.x, acc.y);
      o.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(out_bf16 + r * ld_out + c) = o;
    }
  }
}

// ------------------------------------------------------------------------------ tensor parallel
struct TpReduce {
  int* hdr;                                // this rank's header
  const float* inbox;                      // this rank's inbox [P][cap][H]
  __nv_bfloat16* out;                      // [N, H]
  __nv_bfloat16* gather[LB_PEER_MAX];      // every rank's gather region [cap][H]
  int* peer_hdr[LB_PEER_MAX];
  int P, rank, N, H;
  long long cap;
  int* status;
};

// Rows of the 128-row tiles this rank owns (tile m -> rank m % P): the P partials summed
// in rank order in fp32, rounded once to bf16, written to out and to every other rank's
// gather region (NVLink stores).  The last CTA publishes the epoch to the other ranks.
__global__ void __launch_bounds__(256) k_tp_reduce(const TpReduce a) {
  pdl_entry();
  if ((int)threadIdx.x < a.P) peer_wait(a.hdr + TPH_PART + threadIdx.x, a.hdr[TPH_EPOCH], a.status);
  __syncthreads();
  const int nmt = (a.N + GEMM_BM - 1) / GEMM_BM;
  const int owned = nmt > a.rank ? (nmt - a.rank + a.P - 1) / a.P : 0;
  const int vpr = a.H / 8;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  // one warp per owned row: q-th owned row = row q % 128 of the (q / 128)-th owned tile
  for (int q = blockIdx.x * wpb + (int)(threadIdx.x >> 5); q < owned * GEMM_BM;
       q += gridDim.x * wpb) {
    const int row = (a.rank + a.P * (q / GEMM_BM)) * GEMM_BM + q % GEMM_BM;
    if (row >= a.N) continue;
    for (int c = lane; c < vpr; c += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < a.P; ++s) {
        const float4* src =
            reinterpret_cast<const float4*>(a.inbox + ((long long)s * a.cap + row) * a.H) + 2 * c;
        const float4 x0 = src[0], x1 = src[1];
        acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
        acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
      }
      const uint4 o = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                 pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      reinterpret_cast<uint4*>(a.out + (long long)row * a.H)[c] = o;
      for (int p = 0; p < a.P; ++p)
        if (p != a.rank) reinterpret_cast<uint4*>(a.gather[p] + (long long)row * a.H)[c] = o;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.hdr + TPH_DONE_RED, 1) == (int)gridDim.x - 1) {
    __threadfence_system();
    const int epoch = a.hdr[TPH_EPOCH];
    a.hdr[TPH_DONE_RED] = 0;
    for (int p = 0; p < a.P; ++p)
      if (p != a.rank) st_release_sys(a.peer_hdr[p] + TPH_GATH + a.rank, epoch);
  }
}

// Waits for every other rank's reduced rows, then copies the rows they own into out.
__global__ void __launch_bounds__(256) k_tp_gather(int* hdr, const __nv_bfloat16* __restrict__ gather,
                                                   __nv_bfloat16* __restrict__ out, int P, int rank,
                                                   int N, int H, int* status) {
  pdl_entry();
  if ((int)threadIdx.x < P && (int)threadIdx.x != rank)
    peer_wait(hdr + TPH_GATH + threadIdx.x, hdr[TPH_EPOCH], status);
  __syncthreads();
  const int vpr = H / 8;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  // one warp per row
  for (int row = blockIdx.x * wpb + (int)(threadIdx.x >> 5); row < N; row += gridDim.x * wpb) {
    if ((row / GEMM_BM) % P == rank) continue;
    const uint4* src = reinterpret_cast<const uint4*>(gather + (long long)row * H);
    uint4* dst = reinterpret_cast<uint4*>(out + (long long)row * H);
#pragma unroll 8
    for (int c = lane; c < vpr; c += 32) dst[c] = src[c];
  }
}

// ------------------------------------------------------------------------------ host
struct PodPlan {
  int split_tokens, max_splits, max_ctx, pf_cap, dec_cap, gqa, grid, n_pf_ctas;
  // o_proj: one bf16 GEMM when its output tiles fill the SMs (oproj_direct), else K split
  // oproj_splits ways into fp32 slices that k_splitk_reduce adds in split order
  int oproj_direct, oproj_splits;
};

struct PodWs {
  int* status;
  int* counters;        // [8]: prefill count / next, decode count / next, prologue next / done
  int* seq_ready;       // [B] fused prologue: new tokens stored per sequence
  int4* pf_items;
  int4* dec_items;
  float* part_o;
  float* part_lse;
  __nv_bfloat16* ogated;
  float* o32;
};

// Argument checks of the prologue (standalone lb_attn_prologue or fused into the POD call).
static int check_prologue(const LbPrologueArgs* a) {
  LB_REQUIRE(a != nullptr, "lb_attn_prologue: null args");
  LB_REQUIRE(a->head_dim == POD_D, "lb_attn_prologue: head_dim must be 256");
  LB_REQUIRE(a->num_tokens >= 0 && a->num_q_heads > 0 && a->num_kv_heads > 0 &&
                 a->num_tokens * (a->num_q_heads + a->num_kv_heads) < (1ll << 31),
             "lb_attn_prologue: bad sizes");
  LB_REQUIRE(a->rotary_dim >= 0 && a->rotary_dim <= a->head_dim && a->rotary_dim % 16 == 0,
             "lb_attn_prologue: rotary_dim must be a multiple of 16 and <= head_dim");
  LB_REQUIRE(a->q_in && a->k_in && a->v_in && a->q_norm_w && a->k_norm_w && a->positions &&
                 a->slot_mapping && a->k_cache && a->v_cache && a->q_out &&
                 (a->rotary_dim == 0 || a->cos_sin_cache),
             "lb_attn_prologue: null pointer");
  LB_REQUIRE(a->max_position > 0 && a->num_slots >= 0, "lb_attn_prologue: bad cache sizes");
  LB_REQUIRE(aligned16(a->q_in) && aligned16(a->k_in) && aligned16(a->v_in) &&
                 aligned16(a->q_norm_w) && aligned16(a->k_norm_w) && aligned16(a->k_cache) &&
                 aligned16(a->v_cache) && aligned16(a->q_out),
             "lb_attn_prologue: tensors must be 16-byte aligned");
  LB_REQUIRE(a->q_in_stride_tok % 8 == 0 && a->q_in_stride_head % 8 == 0 &&
                 a->k_in_stride_tok % 8 == 0 && a->v_in_stride_tok % 8 == 0 &&
                 a->q_out_stride_tok % 8 == 0 && a->q_out_stride_head % 8 == 0,
             "lb_attn_prologue: strides must be multiples of 8 elements");
  return LB_OK;
}

static int pod_plan_host(const LbPodArgs* a, PodPlan& pl) {
  LB_REQUIRE(a != nullptr, "lb_pod: null args");
  LB_REQUIRE(a->head_dim == POD_D, "lb_pod: head_dim must be 256 (got %lld)", (long long)a->head_dim);
  LB_REQUIRE(a->num_seqs >= 0 && a->num_seqs <= 16000 && a->num_tokens >= 0 &&
                 a->num_tokens <= (1 << 24),
             "lb_pod: num_seqs/num_tokens out of range");
  LB_REQUIRE(a->num_q_heads > 0 && a->num_kv_heads > 0 && a->num_q_heads % a->num_kv_heads == 0 &&
                 a->num_q_heads / a->num_kv_heads <= 16,
             "lb_pod: need Hq %% Hkv == 0 and Hq/Hkv <= 16");
  LB_REQUIRE(a->page_size > 0 && a->page_size % POD_KV == 0,
             "lb_pod: page_size must be a multiple of 128");
  LB_REQUIRE(a->num_pages > 0 && a->max_pages_per_seq > 0, "lb_pod: empty KV pool / tables");
  LB_REQUIRE(a->num_pages * a->page_size < (1ll << 31), "lb_pod: KV pool too large for 32-bit slots");
  LB_REQUIRE(a->w_o == nullptr || (a->hidden > 0 && a->hidden % 32 == 0),
             "lb_pod: hidden must be a multiple of 32");
  LB_REQUIRE(a->q && a->k_cache && a->v_cache && a->block_tables && a->context_lens &&
                 a->cu_seqlens_q,
             "lb_pod: null pointer");
  LB_REQUIRE((a->w_o && a->out) || (!a->w_o && a->attn_out),
             "lb_pod: need w_o and out, or (attention only) attn_out without w_o");
  LB_REQUIRE(aligned16(a->q) && (a->gate == nullptr || aligned16(a->gate)) &&
                 aligned16(a->k_cache) && aligned16(a->v_cache) &&
                 (a->w_o == nullptr || aligned16(a->w_o)) && (a->out == nullptr || aligned16(a->out)) &&
                 (a->attn_out == nullptr || aligned16(a->attn_out)),
             "lb_pod: tensors must be 16-byte aligned");
  LB_REQUIRE(a->q_stride_head % 8 == 0 && a->q_stride_tok % 8 == 0 && a->q_stride_head >= POD_D,
             "lb_pod: q strides must be multiples of 8 elements with contiguous heads");
  LB_REQUIRE(a->gate == nullptr || (a->gate_stride_head % 8 == 0 && a->gate_stride_tok % 8 == 0 &&
                                    a->gate_stride_head >= POD_D),
             "lb_pod: gate strides must be multiples of 8 elements with contiguous heads");
  if (a->tp_size > 1) {
    LB_REQUIRE(a->tp_size <= LB_EP_MAX_RANKS && a->tp_rank >= 0 && a->tp_rank < a->tp_size,
               "lb_pod: need 1 < tp_size <= %d and 0 <= tp_rank < tp_size", LB_EP_MAX_RANKS);
    LB_REQUIRE(a->w_o && !a->out_fp32 && a->hidden % 256 == 0,
               "lb_pod: tensor parallel o_proj needs w_o, a bf16 out and hidden % 256 == 0");
    LB_REQUIRE(a->tp_capacity >= a->num_tokens, "lb_pod: num_tokens exceeds tp_capacity");
    LB_REQUIRE((a->tp_phases & ~7) == 0, "lb_pod: unknown tp_phases bits");
    for (int r = 0; r < a->tp_size; ++r)
      LB_REQUIRE(a->tp_bufs[r] && (reinterpret_cast<uintptr_t>(a->tp_bufs[r]) & 255) == 0,
                 "lb_pod: tp buffer %d missing or not 256-byte aligned", r);
  }
  if (a->prologue) {
    const LbPrologueArgs* r = a->prologue;
    if (int rc = check_prologue(r)) return rc;
    LB_REQUIRE(r->num_tokens == a->num_tokens && r->num_q_heads == a->num_q_heads &&
                   r->num_kv_heads == a->num_kv_heads,
               "lb_pod: the fused prologue must cover the call's tokens and heads");
    LB_REQUIRE(r->q_out == a->q && r->q_out_stride_tok == a->q_stride_tok &&
                   r->q_out_stride_head == a->q_stride_head,
               "lb_pod: the fused prologue's q_out must be the attention's q");
    LB_REQUIRE(r->k_cache == a->k_cache && r->v_cache == a->v_cache &&
                   r->num_slots == a->num_pages * a->page_size,
               "lb_pod: the fused prologue must store into the attention's paged cache");
  }
  const long long HD = a->num_q_heads * POD_D;
  LB_REQUIRE(HD % 64 == 0, "lb_pod: Hq*D must be a multiple of 64");
  pl.gqa = (int)(a->num_q_heads / a->num_kv_heads);
  pl.max_ctx = (int)std::min<long long>(a->max_pages_per_seq * a->page_size, 1ll << 30);
  const int nsm = num_sms();
  long long split = a->kv_split_pages > 0 ? (long long)a->kv_split_pages * a->page_size : 0;
  if (split == 0) {
    // largest power-of-two page count (<= 16 pages) that still gives every SM about one
    // and a half items: each item pays a fixed start-up and epilogue cost (Q load, split
    // flush, one more partial to merge), so items are made as long as the balance across
    // SMs allows; the planner orders them longest first, which keeps the dynamic tail
    // short.  (A sweep on B200: 64 decode sequences of U[512,4096] tokens take 88.8 us
    // per call with 8-page splits, 92.0 with 4, 99.9 with 2; 128 of U[256,8192] next to a
    // prefill chunk the same 303-304 us with 8 or 16.)  The typical context is the
    // caller's decode-token hint per sequence, else half the table width.
    long long est_ctx = std::max<long long>(1, pl.max_ctx / 2);
    if (a->decode_tokens_hint > 0 && a->num_seqs > 0)
      est_ctx = std::max<long long>(1, a->decode_tokens_hint / a->num_seqs);
    long long pages = 1;
    for (long long pg = 16; pg >= 1; pg >>= 1) {
      const long long st = pg * a->page_size;
      const long long items = a->num_seqs * a->num_kv_heads * ((est_ctx + st - 1) / st);
      if (2 * items >= 3ll * nsm) { pages = pg; break; }
    }
    split = pages * a->page_size;
  }
  pl.split_tokens = (int)split;
  pl.max_splits = (int)((pl.max_ctx + split - 1) / split);
  pl.dec_cap = (int)std::min<long long>(a->num_seqs * a->num_kv_heads * pl.max_splits, 1ll << 30);
  pl.pf_cap = (int)std::min<long long>(a->num_q_heads * ((a->num_tokens + POD_KV - 1) / POD_KV + a->num_seqs),
                                       1ll << 30);
  pl.grid = nsm;
  pl.n_pf_ctas = a->max_q_len > 1 ? nsm / 2 : 0;
  if (a->max_q_len > 1) {
    // Starting split of the SMs between the queues (CTAs that finish their queue switch
    // to the other, so this only sets where they start).  Work is counted in SM-seconds
    // at the per-SM rates this kernel reaches on B200: prefill ~5.5 TFLOP/s per SM,
    // decode ~60 GB/s of KV per SM, with decode as a whole capped at ~6.9 TB/s of HBM.
    // The prefill CTAs get the share that finishes their queue when the decode queue is
    // done, plus 10% so that decode CTAs, not the long prefill tiles, form the tail.
    double pf_pairs = (double)a->prefill_pairs_hint, dec_tok = (double)a->decode_tokens_hint;
    if (pf_pairs <= 0 && dec_tok <= 0) {
      const double pf_rows = (double)std::max<long long>(0, a->num_tokens - (a->num_seqs - 1));
      pf_pairs = pf_rows * (pl.max_ctx / 4.0);
      dec_tok = (double)(a->num_seqs - 1) * (pl.max_ctx / 2.0);
    }
    const double w_pf = pf_pairs * a->num_q_heads * POD_D * 4.0 / 5.5e12;
    const double dec_bytes = dec_tok * a->num_kv_heads * POD_D * 4.0;
    const double w_dec = dec_bytes / 60.0e9;
    const double t_end = std::max(dec_bytes / 6.9e12, (w_pf + w_dec) / nsm);
    const int n = (int)(1.1 * w_pf / std::max(t_end, 1e-9) + 0.5);
    pl.n_pf_ctas = std::max(1, std::min(nsm, n));
  }
  pl.oproj_direct = 1;
  pl.oproj_splits = 1;
  if (a->w_o && a->tp_size <= 1) {
    const long long K = a->num_q_heads * POD_D, Hd = a->hidden;
    const long long mt = (a->num_tokens + GEMM_BM - 1) / GEMM_BM;
    const long long tiles = mt * (Hd / ((Hd % 128 == 0) ? 128 : 32));
    if (a->out_fp32 || tiles * 2 < nsm) {
      pl.oproj_direct = 0;
      const int kb = (int)(K / 64);
      while (pl.oproj_splits * 2 <= kb && kb % (pl.oproj_splits * 2) == 0 &&
             tiles * pl.oproj_splits * 2 <= nsm)
        pl.oproj_splits *= 2;
    }
  }
  return LB_OK;
}

static size_t carve_pod(const LbPodArgs& a, const PodPlan& pl, void* base, PodWs& w) {
  Carve c(base, ~size_t(0));
  w.status = c.take<int>(64);
  w.counters = c.take<int>(8);
  w.seq_ready = c.take<int>(a.prologue ? (size_t)a.num_seqs : 0);
  w.pf_items = c.take<int4>(pl.pf_cap);
  w.dec_items = c.take<int4>(pl.dec_cap);
  w.part_o = c.take<float>((size_t)a.num_seqs * pl.max_splits * a.num_q_heads * POD_D);
  w.part_lse = c.take<float>((size_t)a.num_seqs * pl.max_splits * a.num_q_heads);
  w.ogated = c.take<__nv_bfloat16>((size_t)a.num_tokens * a.num_q_heads * POD_D);
  w.o32 = c.take<float>(a.w_o && !pl.oproj_direct
                            ? (size_t)a.num_tokens * a.hidden * pl.oproj_splits : 0);
  return c.off + 256;
}

// Plan, POD attention kernel and split merge (+ gate): writes the o_proj input rows.
static int pod_attention(const LbPodArgs& a, const PodPlan& pl, const PodWs& w, cudaStream_t st) {
  const int B = (int)a.num_seqs, N = (int)a.num_tokens;
  if (B == 0 || N == 0) return LB_OK;
  int rc;
  // TMA maps.  K/V: [slots, Hkv, D] boxes of 128 slots x 1 head x 64 dims.  Q: [N, Hq, D];
  // decode box = 16 heads x 64 dims of one token, prefill box = 128 tokens of one head.
  CUtensorMap tmK, tmV, tmK64, tmV64, tmQd, tmQp;
  const int qd_rows = (int)std::min<long long>(16, a.num_q_heads);
  {
    const uint64_t slots = (uint64_t)(a.num_pages * a.page_size);
    if ((rc = make_tmap_bf16_3d_box(&tmK, a.k_cache, slots, a.num_kv_heads, POD_D,
                                    (uint64_t)a.num_kv_heads * POD_D, POD_D, POD_KV, 1, 64)))
      return rc;
    if ((rc = make_tmap_bf16_3d_box(&tmV, a.v_cache, slots, a.num_kv_heads, POD_D,
                                    (uint64_t)a.num_kv_heads * POD_D, POD_D, POD_KV, 1, 64)))
      return rc;
    if ((rc = make_tmap_bf16_3d_box(&tmK64, a.k_cache, slots, a.num_kv_heads, POD_D,
                                    (uint64_t)a.num_kv_heads * POD_D, POD_D, PF_KV, 1, 64)))
      return rc;
    if ((rc = make_tmap_bf16_3d_box(&tmV64, a.v_cache, slots, a.num_kv_heads, POD_D,
                                    (uint64_t)a.num_kv_heads * POD_D, POD_D, PF_KV, 1, 64)))
      return rc;
    if ((rc = make_tmap_bf16_3d_box(&tmQd, a.q, N, a.num_q_heads, POD_D, a.q_stride_tok,
                                    a.q_stride_head, 1, qd_rows, 64)))
      return rc;
    if ((rc = make_tmap_bf16_3d_box(&tmQp, a.q, N, a.num_q_heads, POD_D, a.q_stride_tok,
                                    a.q_stride_head, POD_KV, 1, 64)))
      return rc;
  }
  if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(k_pod_plan), (int)(3 * sizeof(int) * B))))
    return rc;
  launch_k(k_pod_plan, 1, 1024, 3 * sizeof(int) * B, st, a.context_lens, a.cu_seqlens_q, B, (int)a.num_q_heads,
                                 (int)a.num_kv_heads, pl.split_tokens, pl.max_splits, pl.max_ctx,
                                 pl.pf_cap, pl.dec_cap, w.pf_items, w.counters, w.dec_items,
                                 a.prologue ? w.seq_ready : nullptr, w.status);
  { int _rc = launched("k_pod_plan"); if (_rc) return _rc; }

  PodParams p{};
  p.status = w.status;
  p.pf_items = w.pf_items;
  p.pf_count = w.counters + 0;
  p.pf_next = w.counters + 1;
  p.dec_items = w.dec_items;
  p.dec_count = w.counters + 2;
  p.dec_next = w.counters + 3;
  p.block_tables = a.block_tables;
  p.bt_stride = a.max_pages_per_seq;
  p.context_lens = a.context_lens;
  p.cu_seqlens_q = a.cu_seqlens_q;
  p.gate = static_cast<const __nv_bfloat16*>(a.gate);
  p.gate_st = a.gate_stride_tok;
  p.gate_sh = a.gate_stride_head;
  p.ogated = a.w_o ? w.ogated : nullptr;
  p.attn_out = static_cast<__nv_bfloat16*>(a.attn_out);
  p.part_o = w.part_o;
  p.part_lse = w.part_lse;
  p.max_splits = pl.max_splits;
  p.Hq = (int)a.num_q_heads;
  p.Hkv = (int)a.num_kv_heads;
  p.gqa = pl.gqa;
  p.page_size = (int)a.page_size;
  p.num_pages = (int)a.num_pages;
  p.split_tokens = pl.split_tokens;
  p.n_prefill_ctas = pl.n_pf_ctas;
  p.scale_log2 = a.sm_scale * 1.4426950408889634f;
  p.qd_bytes = 4 * qd_rows * 128;
  p.num_tokens = N;
  p.num_seqs = B;
  if (a.prologue) {
    p.pro = *a.prologue;
    p.pro_tasks = (N + PRO_TASK_TOKENS - 1) / PRO_TASK_TOKENS;
    p.pro_next = w.counters + 4;
    p.pro_done = w.counters + 5;
    p.seq_ready = w.seq_ready;
  }
  if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(k_pod_attn), POD_SMEM))) return rc;
  record_event(a.timing_events[0], st);
  launch_k(k_pod_attn, pl.grid, POD_THREADS, POD_SMEM, st, tmK, tmV, tmK64, tmV64, tmQd, tmQp, p);
  { int _rc = launched("k_pod_attn"); if (_rc) return _rc; }
  record_event(a.timing_events[1], st);

  // heads per merge CTA: all of them when the sequences alone give every SM two CTAs,
  // else 4 (128 threads, 8 dims each) when Hq allows, for more CTAs in flight
  const int hpc = (B >= 2ll * num_sms() || a.num_q_heads % 4 != 0) ? (int)a.num_q_heads : 4;
  const size_t merge_smem = sizeof(float) * (size_t)pl.max_splits * hpc;
  LB_REQUIRE(merge_smem <= 48 * 1024, "lb_pod: too many decode splits (%d)", pl.max_splits);
  const long long merge_grid = B * (a.num_q_heads / hpc);
  LB_REQUIRE(merge_grid < (1ll << 31), "lb_pod: too many sequences x heads");
  launch_k(k_pod_merge, (int)merge_grid, std::min(256, 32 * hpc), merge_smem, st, a.context_lens,
                                          a.cu_seqlens_q, (int)a.num_q_heads, hpc,
                                          pl.split_tokens, pl.max_splits, pl.max_ctx, w.part_o,
                                          w.part_lse, p.gate, a.gate_stride_tok, a.gate_stride_head,
                                          p.ogated, p.attn_out);
  { int _rc = launched("k_pod_merge"); if (_rc) return _rc; }
  return LB_OK;
}

// Tensor-parallel o_proj: GEMM with the peer-store epilogue, owner reduction, gather.
static int tp_oproj(const LbPodArgs& a, const PodWs& w, cudaStream_t st, int phases) {
  const int N = (int)a.num_tokens, P = a.tp_size, rank = a.tp_rank;
  const int K = (int)(a.num_q_heads * POD_D), Hd = (int)a.hidden;
  const int nsm = num_sms();
  TpPeers tp{};
  for (int r = 0; r < P; ++r) {
    uint8_t* base = static_cast<uint8_t*>(a.tp_bufs[r]);
    tp.hdr[r] = reinterpret_cast<int*>(base);
    tp.inbox[r] = reinterpret_cast<float*>(base + TP_HEADER_BYTES);
  }
  tp.rank = rank;
  tp.size = P;
  tp.inbox_rows = a.tp_capacity;
  uint8_t* own = static_cast<uint8_t*>(a.tp_bufs[rank]);
  int* hdr = tp.hdr[rank];
  const size_t inbox_bytes = (size_t)P * a.tp_capacity * Hd * sizeof(float);
  auto gather_of = [&](int r) {
    return reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(a.tp_bufs[r]) + TP_HEADER_BYTES +
                                            inbox_bytes);
  };
  int rc;
  if (phases & LB_TP_PHASE_ATTN) {
    constexpr int BN = 256;
    CUtensorMap tA, tB;
    // an empty rank still launches (its CTAs publish the epoch); its maps point at W_o
    const void* A = N > 0 ? static_cast<const void*>(w.ogated) : a.w_o;
    if ((rc = make_tmap_bf16_2d(&tA, A, std::max(N, 1), K, K, GEMM_BM, 64))) return rc;
    if ((rc = make_tmap_bf16_3d(&tB, a.w_o, 1, Hd, K, K, (uint64_t)K * Hd, BN, 64))) return rc;
    GemmArgs g = gemm_args_default(w.status);
    g.m = N;
    g.n_tiles = Hd / BN;
    g.splits = 1;
    g.k_blocks = K / 64;
    g.out = nullptr;
    g.ldo = Hd;
    g.out_rows = N;
    g.out_cols = Hd;
    g.tp = tp;
    const long long tiles = (long long)((N + GEMM_BM - 1) / GEMM_BM) * g.n_tiles;
    const int grid = (int)std::max<long long>(1, std::min<long long>(tiles, nsm));
    record_event(a.timing_events[2], st);
    if ((rc = launch_gemm<BN, 4, EPI_F32_PEER>(tA, tB, g, grid, st))) return rc;
  }
  if (phases & LB_TP_PHASE_REDUCE) {
    TpReduce d{};
    d.hdr = hdr;
    d.inbox = reinterpret_cast<const float*>(own + TP_HEADER_BYTES);
    d.out = static_cast<__nv_bfloat16*>(a.out);
    for (int r = 0; r < P; ++r) {
      d.gather[r] = gather_of(r);
      d.peer_hdr[r] = tp.hdr[r];
    }
    d.P = P;
    d.rank = rank;
    d.N = N;
    d.H = Hd;
    d.cap = a.tp_capacity;
    d.status = w.status;
    const long long units = (long long)N * (Hd / 8) / P + Hd;
    const int grid = (int)std::max<long long>(1, std::min<long long>(nsm * 2, (units + 255) / 256));
    launch_k(k_tp_reduce, grid, 256, 0, st, d);
    { int _rc = launched("k_tp_reduce"); if (_rc) return _rc; }
  }
  if (phases & LB_TP_PHASE_GATHER) {
    const long long units = (long long)N * (Hd / 8);
    const int grid = (int)std::max<long long>(1, std::min<long long>(nsm * 2, (units + 255) / 256));
    launch_k(k_tp_gather, grid, 256, 0, st, hdr, gather_of(rank), static_cast<__nv_bfloat16*>(a.out), P,
                                       rank, N, Hd, w.status);
    { int _rc = launched("k_tp_gather"); if (_rc) return _rc; }
    record_event(a.timing_events[3], st);
  }
  return LB_OK;
}

static int pod_run(const LbPodArgs& a, const PodPlan& pl, const PodWs& w, cudaStream_t st) {
  const bool tp = a.tp_size > 1;
  const int phases = (tp && a.tp_phases) ? a.tp_phases : 7;
  int rc;
  if (phases & LB_TP_PHASE_ATTN) {
    if ((rc = pod_attention(a, pl, w, st))) return rc;
  }
  if (a.w_o == nullptr) return LB_OK;  // attention only
  if (tp) return tp_oproj(a, w, st, phases);
  const int N = (int)a.num_tokens;
  if (a.num_seqs == 0 || N == 0) return LB_OK;
  // o_proj: out[N, hidden] = ogated[N, Hq*D] . W_o^T
  const int K = (int)(a.num_q_heads * POD_D), Hd = (int)a.hidden;
  const int nsm = num_sms();
  record_event(a.timing_events[2], st);
  if (pl.oproj_direct) {
    rc = gemm_run(w.ogated, K, a.w_o, K, a.out, Hd, N, Hd, K, EPI_BF16, 1, w.status, st);
    record_event(a.timing_events[3], st);
    return rc;
  }
  // few output tiles: K split over the SMs, each split's fp32 partial in its own slice,
  // the slices added in split order (no atomics, no zeroing: a deterministic result)
  const int splits = pl.oproj_splits;
  rc = gemm_run(w.ogated, K, a.w_o, K, w.o32, Hd, N, Hd, K, EPI_F32_SPLIT, splits, w.status, st);
  if (rc) return rc;
  const int g = (int)std::max<long long>(1, std::min<long long>(nsm * 8, (N * (Hd / 4) + 255) / 256));
  launch_k(k_splitk_reduce, g, 256, 0, st, static_cast<const float*>(w.o32), splits, (long long)N,
           Hd, a.out_fp32 ? nullptr : static_cast<__nv_bfloat16*>(a.out),
           a.out_fp32 ? static_cast<float*>(a.out) : nullptr, (long long)Hd);
  { int _rc = launched("k_splitk_reduce"); if (_rc) return _rc; }
  record_event(a.timing_events[3], st);
  return LB_OK;
}
}  // namespace lb

using namespace lb;

extern "C" {

int lb_store_kvcache(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                     void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t N,
                     int64_t num_slots, int64_t row_elems, void* stream) {
  LB_REQUIRE(k && v && k_cache && v_cache && slot_mapping, "lb_store_kvcache: null pointer");
  LB_REQUIRE(N >= 0 && row_elems > 0 && row_elems % 8 == 0 && k_stride % 8 == 0 &&
                 v_stride % 8 == 0,
             "lb_store_kvcache: rows must be multiples of 8 elements");
  LB_REQUIRE(aligned16(k) && aligned16(v) && aligned16(k_cache) && aligned16(v_cache),
             "lb_store_kvcache: unaligned pointer");
  if (N == 0) return LB_OK;
  const int threads = 256;
  const long long blocks = (N * 32 + threads - 1) / threads;
  launch_k(k_store_kvcache, (unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(k), k_stride, static_cast<const __nv_bfloat16*>(v),
      v_stride, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
      slot_mapping, (int)N, num_slots, (int)row_elems);
  { int _rc = launched("k_store_kvcache"); if (_rc) return _rc; }
  return LB_OK;
}

int lb_attn_prologue(const LbPrologueArgs* a, void* stream) {
  if (int rc = check_prologue(a)) return rc;
  if (a->num_tokens == 0) return LB_OK;
  const long long tasks = (a->num_tokens + PRO_TASK_TOKENS - 1) / PRO_TASK_TOKENS;
  const long long blocks = std::max<long long>(1, std::min<long long>(tasks, num_sms() * 8));
  launch_k(k_attn_prologue, (unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream), *a);
  { int _rc = launched("k_attn_prologue"); if (_rc) return _rc; }
  return LB_OK;
}

size_t lb_tp_buffer_size(int64_t world, int64_t capacity, int64_t hidden) {
  if (world < 1 || capacity < 0 || hidden < 0) return 0;
  return (size_t)TP_HEADER_BYTES + (size_t)world * capacity * hidden * sizeof(float) +
         (size_t)capacity * hidden * sizeof(__nv_bfloat16) + 256;
}

int lb_pod_workspace_size(const LbPodArgs* a, size_t* bytes) {
  PodPlan pl;
  int rc = pod_plan_host(a, pl);
  if (rc) return rc;
  LB_REQUIRE(bytes != nullptr, "lb_pod_workspace_size: null output");
  PodWs w;
  *bytes = carve_pod(*a, pl, nullptr, w);
  return LB_OK;
}

int lb_pod_attn_oproj(const LbPodArgs* a, void* stream) {
  PodPlan pl;
  int rc = pod_plan_host(a, pl);
  if (rc) return rc;
  PodWs w;
  const size_t need = carve_pod(*a, pl, a->workspace, w);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(LB_ERR_WORKSPACE, "lb_pod_attn_oproj: workspace %zu < %zu bytes",
                (size_t)a->workspace_bytes, need);
  return pod_run(*a, pl, w, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
