// The full-attention prologue after the projections, as device code shared by the
// standalone kernel (lb_attn_prologue) and the POD attention kernel's first phase:
// for token n, query head h and KV head g,
//   q_out[n, h]          = RoPE(RMSNorm_1pw(q_in[n, h], q_norm_w))
//   k_cache[slot[n], g]  = RoPE(RMSNorm_1pw(k_in[n, g], k_norm_w))
//   v_cache[slot[n], g]  = v_in[n, g]
// (nanovllm/models/qwen3_5.py:39-55, 707-736; rotary_embedding.py:5-54; store_kvcache,
// attention.py:50-80).  The RMSNorm and RoPE follow the reference's fp32 operation order
// with explicit rounding (no contraction), so the bf16 results match it up to the order
// of the sum of squares.
//
// Work is cut into tasks of PRO_TASK_TOKENS tokens that one thread block does together:
// it first stages the tokens' cache slots and cos/sin rows in shared memory, then its
// warps take the task's rows -- Hq query rows, Hkv key rows and Hkv value rows per token,
// one warp per row of D = 256 dims, a lane holding 8 consecutive dims -- in batches whose
// loads are all issued before any is used (one independent 512-byte load per row).
#pragma once

#include <cuda_bf16.h>

#include "../../include/layerbatch_b200.h"
#include "lb_common.cuh"

namespace lb {

constexpr int PRO_D = 256;            // head_dim the prologue handles
constexpr int PRO_TASK_TOKENS = 16;   // tokens of one task
constexpr int PRO_BATCH = 8;          // rows a warp loads before it uses any

// Per-task staging area in shared memory.
struct ProStage {
  int tok[PRO_TASK_TOKENS];               // the task's tokens, -1: none (invalid entry)
  int slot[PRO_TASK_TOKENS];              // cache slot of each token, -1: nothing to store
  float cs[PRO_TASK_TOKENS][PRO_D];       // cos | sin row of each token's position
};

// One loaded row.  Token indices fit 32 bits (the callers check N).
struct ProRow {
  uint4 x;    // this lane's 8 dims of the row
  int n;      // token within the task
  int h;      // row kind and head: [0, Hq) query, [Hq, Hq+Hkv) key, then value; -1: none
};

__device__ __forceinline__ ProRow prologue_load(const LbPrologueArgs& a, const ProStage* st,
                                                int n, int h, int lane) {
  ProRow r;
  r.n = n;
  r.h = h;
  r.x = make_uint4(0, 0, 0, 0);
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  const long long t = st->tok[n];
  if (t < 0) {
    r.h = -1;
    return r;
  }
  const __nv_bfloat16* src;
  if (h < Hq) {
    src = static_cast<const __nv_bfloat16*>(a.q_in) + t * a.q_in_stride_tok +
          (long long)h * a.q_in_stride_head;
  } else {
    if (st->slot[n] < 0) {   // padding token or a slot outside the cache: no store
      r.h = -1;
      return r;
    }
    src = h < Hq + Hkv
              ? static_cast<const __nv_bfloat16*>(a.k_in) + t * a.k_in_stride_tok +
                    (long long)(h - Hq) * PRO_D
              : static_cast<const __nv_bfloat16*>(a.v_in) + t * a.v_in_stride_tok +
                    (long long)(h - Hq - Hkv) * PRO_D;
  }
  r.x = reinterpret_cast<const uint4*>(src)[lane];
  return r;
}

// The (1 + w) factors of the two norms for this lane's 8 dims, once per task.
struct ProNorm {
  float q[8], k[8];
};

__device__ __forceinline__ ProNorm prologue_norm(const LbPrologueArgs& a, int lane) {
  ProNorm w;
  const uint4 qw = reinterpret_cast<const uint4*>(a.q_norm_w)[lane];
  const uint4 kw = reinterpret_cast<const uint4*>(a.k_norm_w)[lane];
  const uint32_t qv[4] = {qw.x, qw.y, qw.z, qw.w}, kv[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w.q[2 * i] = __fadd_rn(1.0f, bf16_lo(qv[i]));
    w.q[2 * i + 1] = __fadd_rn(1.0f, bf16_hi(qv[i]));
    w.k[2 * i] = __fadd_rn(1.0f, bf16_lo(kv[i]));
    w.k[2 * i + 1] = __fadd_rn(1.0f, bf16_hi(kv[i]));
  }
  return w;
}

// The normalised (and, for the first rotary_dim dims, rotated) bf16 row of a loaded query
// or key row, this lane's 8 dims packed.  All 32 lanes of the warp call it together (warp
// shuffles).  `cs` is the row's cos|sin table row; only the lanes holding rotated dims read
// it.  The normalised row is rounded to bf16 before the rotation, as the reference rounds
// the norm's output.
__device__ __forceinline__ uint4 prologue_row_math(const LbPrologueArgs& a, const uint4& xr,
                                                   bool is_q, const float* cs, int lane,
                                                   const ProNorm& nw) {
  const uint32_t xv[4] = {xr.x, xr.y, xr.z, xr.w};
  float x[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = bf16_lo(xv[i]);
    x[2 * i + 1] = bf16_hi(xv[i]);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float rstd = rsqrtf(__fadd_rn(ss / (float)PRO_D, a.eps));
  uint32_t yb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float w0 = is_q ? nw.q[2 * i] : nw.k[2 * i];
    const float w1 = is_q ? nw.q[2 * i + 1] : nw.k[2 * i + 1];
    yb[i] = pack_bf16x2(__fmul_rn(__fmul_rn(x[2 * i], rstd), w0),
                        __fmul_rn(__fmul_rn(x[2 * i + 1], rstd), w1));
  }
  // partial RoPE: dims [0, rot/2) pair with [rot/2, rot); lanes < rot/16 hold the first
  // half, the next rot/16 lanes the second
  const int rot = (int)a.rotary_dim;
  const int hl = rot / 16;
  const bool first = lane < hl, second = lane >= hl && lane < 2 * hl;
  const int partner = first ? lane + hl : (second ? lane - hl : lane);
  uint32_t pb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) pb[i] = __shfl_sync(0xffffffffu, yb[i], partner);
  if (first || second) {
    const int f0 = (first ? lane : lane - hl) * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float y2[2] = {bf16_lo(yb[i]), bf16_hi(yb[i])};
      const float p2[2] = {bf16_lo(pb[i]), bf16_hi(pb[i])};
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float c = cs[f0 + 2 * i + u], sn = cs[rot / 2 + f0 + 2 * i + u];
        y2[u] = first ? __fsub_rn(__fmul_rn(y2[u], c), __fmul_rn(p2[u], sn))   // x1 c - x2 s
                      : __fadd_rn(__fmul_rn(y2[u], c), __fmul_rn(p2[u], sn));  // x2 c + x1 s
      }
      yb[i] = pack_bf16x2(y2[0], y2[1]);
    }
  }
  return make_uint4(yb[0], yb[1], yb[2], yb[3]);
}

// Store one row: the query row to q_out, the key row (normalised, rotated) or the value row
// (as loaded) into the cache at `slot`.  h: [0, Hq) query, [Hq, Hq+Hkv) key, then value.
__device__ __forceinline__ void prologue_put(const LbPrologueArgs& a, long long t, int h,
                                             long long slot, const uint4& v, int lane) {
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  if (h < Hq) {
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.q_out) + t * a.q_out_stride_tok +
                         (long long)h * a.q_out_stride_head;
    reinterpret_cast<uint4*>(dst)[lane] = v;
  } else if (h < Hq + Hkv) {
    const long long row = slot * Hkv * PRO_D + (long long)(h - Hq) * PRO_D;
    reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.k_cache) + row)[lane] = v;
  } else {
    const long long row = slot * Hkv * PRO_D + (long long)(h - Hq - Hkv) * PRO_D;
    reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.v_cache) + row)[lane] = v;
  }
}

// A staged row (prologue_task): normalise / rotate query and key rows, store every row.
__device__ __forceinline__ void prologue_store(const LbPrologueArgs& a, const ProStage* st,
                                               const ProRow& r, int lane, const ProNorm& nw) {
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  if (r.h >= Hq + Hkv) {   // value row (a warp-uniform branch: the row is the warp's)
    prologue_put(a, st->tok[r.n], r.h, st->slot[r.n], r.x, lane);
    return;
  }
  const uint4 y = prologue_row_math(a, r.x, r.h < Hq, st->cs[r.n], lane, nw);
  if (r.h >= 0) prologue_put(a, st->tok[r.n], r.h, st->slot[r.n], y, lane);
}

// One task: entries [e0, e0 + ntok) of the token list `toks` (NULL: tokens e0, e0 + 1, ...),
// ntok <= PRO_TASK_TOKENS.  Every thread of the block calls it (it stages with the whole
// block and meets at __syncthreads); `nwarps` warps (warp ids [0, nwarps)) take the rows.
// The caller separates consecutive tasks with a __syncthreads, as the staging area is
// reused.  Tokens outside [0, num_tokens) are reported and skipped.
__device__ __forceinline__ void prologue_task(const LbPrologueArgs& a, const int* toks, int e0,
                                              int ntok, ProStage* st, int warp, int nwarps,
                                              int lane, int* status) {
  const int rot = (int)a.rotary_dim;
  for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
    int t = toks ? toks[e0 + i] : e0 + i;
    if (t < 0 || t >= a.num_tokens) {
      report(status, LB_DEV_BAD_INDEX);
      t = -1;
    }
    st->tok[i] = t;
    const long long s = t < 0 ? -1 : (long long)a.slot_mapping[t];
    if (s >= a.num_slots) report(status, LB_DEV_BAD_INDEX);
    st->slot[i] = (s < 0 || s >= a.num_slots) ? -1 : (int)s;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ntok * rot; e += blockDim.x) {
    const int i = e / rot, c = e - (e / rot) * rot;
    const int t = st->tok[i];
    long long pos = t < 0 ? 0 : a.positions[t];
    if (pos < 0 || pos >= a.max_position) {
      if (c == 0) report(status, LB_DEV_BAD_INDEX);
      pos = pos < 0 ? 0 : a.max_position - 1;
    }
    st->cs[i][c] = a.cos_sin_cache[pos * rot + c];
  }
  __syncthreads();
  if (warp >= nwarps) return;
  const ProNorm nw = prologue_norm(a, lane);
  const int nh = (int)(a.num_q_heads + 2 * a.num_kv_heads);
  const int rows = ntok * nh;
  for (int j0 = warp * PRO_BATCH; j0 < rows; j0 += nwarps * PRO_BATCH) {
    ProRow r[PRO_BATCH];
    int n = j0 / nh, h = j0 - (j0 / nh) * nh;   // row j0; the next rows step the head
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) {
      if (j0 + i < rows) {
        r[i] = prologue_load(a, st, n, h, lane);
      } else {
        r[i].h = -1;
        r[i].n = 0;
        r[i].x = make_uint4(0, 0, 0, 0);
      }
      if (++h == nh) {
        h = 0;
        ++n;
      }
    }
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) prologue_store(a, st, r[i], lane, nw);
  }
}

// Rows of the contiguous tokens [t0, t0 + ntok) loaded straight from global memory (no
// staging: each row reads its token's slot and, on the rotated lanes, its cos/sin row),
// `nwarps` warps from `warp` on, PRO_BATCH rows in flight per warp.  Whole warps call it.
__device__ __forceinline__ void prologue_rows_direct(const LbPrologueArgs& a, int t0, int ntok,
                                                     int warp, int nwarps, int lane,
                                                     const ProNorm& nw, int* status) {
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  const int nh = Hq + 2 * Hkv;
  const int rows = ntok * nh;
  const int rot = (int)a.rotary_dim;
  for (int j0 = warp * PRO_BATCH; j0 < rows; j0 += nwarps * PRO_BATCH) {
    uint4 x[PRO_BATCH];
    int tt[PRO_BATCH], hh[PRO_BATCH], sl[PRO_BATCH];
    int n = j0 / nh, h = j0 - (j0 / nh) * nh;
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) {
      const int t = t0 + n;
      tt[i] = t;
      hh[i] = (j0 + i < rows) ? h : -1;
      sl[i] = 0;
      x[i] = make_uint4(0, 0, 0, 0);
      if (hh[i] >= Hq) {
        const long long s = (long long)a.slot_mapping[t];
        if (s >= a.num_slots) report(status, LB_DEV_BAD_INDEX);
        if (s < 0 || s >= a.num_slots) hh[i] = -1;
        sl[i] = (int)s;
      }
      if (hh[i] >= 0) {
        const __nv_bfloat16* src =
            hh[i] < Hq ? static_cast<const __nv_bfloat16*>(a.q_in) + (long long)t * a.q_in_stride_tok +
                             (long long)hh[i] * a.q_in_stride_head
            : hh[i] < Hq + Hkv ? static_cast<const __nv_bfloat16*>(a.k_in) + (long long)t * a.k_in_stride_tok +
                                     (long long)(hh[i] - Hq) * PRO_D
                               : static_cast<const __nv_bfloat16*>(a.v_in) + (long long)t * a.v_in_stride_tok +
                                     (long long)(hh[i] - Hq - Hkv) * PRO_D;
        x[i] = reinterpret_cast<const uint4*>(src)[lane];
      }
      if (++h == nh) {
        h = 0;
        ++n;
      }
    }
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) {
      if (hh[i] >= Hq + Hkv) {   // value row
        prologue_put(a, tt[i], hh[i], sl[i], x[i], lane);
        continue;
      }
      const float* cs = a.cos_sin_cache;
      if (hh[i] >= 0 && rot > 0 && lane < rot / 8) {
        long long pos = a.positions[tt[i]];
        if (pos < 0 || pos >= a.max_position) {
          report(status, LB_DEV_BAD_INDEX);
          pos = pos < 0 ? 0 : a.max_position - 1;
        }
        cs += pos * rot;
      }
      const uint4 y = prologue_row_math(a, x[i], hh[i] < Hq, cs, lane, nw);
      if (hh[i] >= 0) prologue_put(a, tt[i], hh[i], sl[i], y, lane);
    }
  }
}

// ------------------------------------------------------------------------------ in the GEMM
// The prologue as the epilogue of the q/k/v projection GEMM (EPI_QKV): the GEMM's
// 256-column output tile `ntile` of the stacked weight [q_proj (query | gate per head);
// k_proj; v_proj] is one head row of kind query, gate, key or value for each of the
// tile's 128 tokens; the epilogue thread of a row holds all 256 of its accumulators in
// TMEM.  Query and key rows: rounded to bf16 (the projection's output), (1+w) RMSNorm with
// the sum of squares taken in exactly the order of prologue_row_math (8-dim partial sums,
// then the 32 partials pairwise at distances 16, 8, 4, 2, 1, as the warp's butterfly
// does), the same rounding points, RoPE on the first 64 dims; then the query row goes to
// q_out and the key row into the cache.  Value rows go into the cache as bf16, gate rows
// into the GEMM's own output (where the attention kernel reads the gate).  The stores are
// those of the separate prologue kernel, bit for bit.  rotary_dim must be 64 (the callers
// check it).  All lanes of the warp call this (TMEM loads are warp-collective); `row_ok`
// false: no loads of the token's metadata, no stores.
constexpr int PRO_GEMM_ROT = 64;

__device__ __forceinline__ void pro_ld_row32(uint32_t taddr, float (&x)[32]) {
  uint32_t v[32];
  __syncwarp();
  tmem_ld32(taddr, v);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[i])));
}

__device__ __forceinline__ void pro_store32(__nv_bfloat16* dst, const float (&y)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d[q] = make_uint4(pack_bf16x2(y[8 * q], y[8 * q + 1]), pack_bf16x2(y[8 * q + 2], y[8 * q + 3]),
                      pack_bf16x2(y[8 * q + 4], y[8 * q + 5]), pack_bf16x2(y[8 * q + 6], y[8 * q + 7]));
}

// y = bf16(x * rstd * (1 + w)) for 32 dims starting at d0 of a norm weight row
__device__ __forceinline__ void pro_norm32(float (&x)[32], float rstd, const __nv_bfloat16* nw, int d0) {
  const uint4* wp = reinterpret_cast<const uint4*>(nw + d0);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w4 = wp[q];
    const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float w0 = __fadd_rn(1.0f, bf16_lo(wv[i]));
      const float w1 = __fadd_rn(1.0f, bf16_hi(wv[i]));
      const int e = 8 * q + 2 * i;
      x[e] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[e], rstd), w0)));
      x[e + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[e + 1], rstd), w1)));
    }
  }
}

__device__ __forceinline__ void qkv_prologue_tile(const LbPrologueArgs& a, int ntile, uint32_t tbase,
                                                  bool row_ok, long long t, void* qkv_out,
                                                  long long ldo, int* gemm_status) {
  int* status = a.status ? a.status : gemm_status;
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  int kind, hh;  // 0 query, 1 gate, 2 key, 3 value
  if (ntile < 2 * Hq) {
    hh = ntile >> 1;
    kind = (ntile & 1) ? 1 : 0;
  } else if (ntile < 2 * Hq + Hkv) {
    hh = ntile - 2 * Hq;
    kind = 2;
  } else {
    hh = ntile - 2 * Hq - Hkv;
    kind = 3;
  }
  __nv_bfloat16* dst = nullptr;
  long long pos = 0;
  if (row_ok) {
    if (kind == 1) {
      dst = static_cast<__nv_bfloat16*>(qkv_out) + t * ldo + (long long)ntile * PRO_D;
    } else if (kind == 0) {
      dst = static_cast<__nv_bfloat16*>(a.q_out) + t * a.q_out_stride_tok + (long long)hh * a.q_out_stride_head;
    } else {
      const long long s = (long long)a.slot_mapping[t];
      if (s >= a.num_slots) report(status, LB_DEV_BAD_INDEX);
      if (s >= 0 && s < a.num_slots)
        dst = static_cast<__nv_bfloat16*>(kind == 2 ? a.k_cache : a.v_cache) +
              (s * Hkv + hh) * (long long)PRO_D;
    }
    if (kind == 0 || kind == 2) {
      pos = a.positions[t];
      if (pos < 0 || pos >= a.max_position) {
        if (kind == 0 && hh == 0) report(status, LB_DEV_BAD_INDEX);
        pos = pos < 0 ? 0 : a.max_position - 1;
      }
    }
  }
  if (kind == 1 || kind == 3) {
#pragma unroll 1
    for (int ch = 0; ch < PRO_D / 32; ++ch) {
      float x[32];
      pro_ld_row32(tbase + ch * 32, x);
      if (dst) pro_store32(dst + ch * 32, x);
    }
    return;
  }
  // sum of squares: 32 partials of 8 dims, then the butterfly's pairing
  float part[32];
#pragma unroll
  for (int ch = 0; ch < PRO_D / 32; ++ch) {
    float x[32];
    pro_ld_row32(tbase + ch * 32, x);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(x[8 * g + i], x[8 * g + i]));
      part[4 * ch + g] = ss;
    }
  }
#pragma unroll
  for (int w = 16; w > 0; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) part[i] = __fadd_rn(part[i], part[i + w]);
  const float rstd = rsqrtf(__fadd_rn(part[0] / (float)PRO_D, a.eps));
  const __nv_bfloat16* nw = static_cast<const __nv_bfloat16*>(kind == 0 ? a.q_norm_w : a.k_norm_w);
  {
    // dims [0, 64): norm, then RoPE pairs (i, i + 32)
    float x0[32], x1[32];
    pro_ld_row32(tbase, x0);
    pro_ld_row32(tbase + 32, x1);
    pro_norm32(x0, rstd, nw, 0);
    pro_norm32(x1, rstd, nw, 32);
    const float4* cs = reinterpret_cast<const float4*>(a.cos_sin_cache + pos * PRO_GEMM_ROT);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 c4 = cs[q], s4 = cs[8 + q];
      const float c[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = 4 * q + u;
        const float y1 = x0[i], y2 = x1[i];
        x0[i] = __fsub_rn(__fmul_rn(y1, c[u]), __fmul_rn(y2, sn[u]));
        x1[i] = __fadd_rn(__fmul_rn(y2, c[u]), __fmul_rn(y1, sn[u]));
      }
    }
    if (dst) {
      pro_store32(dst, x0);
      pro_store32(dst + 32, x1);
    }
  }
#pragma unroll 1
  for (int ch = 2; ch < PRO_D / 32; ++ch) {
    float x[32];
    pro_ld_row32(tbase + ch * 32, x);
    pro_norm32(x, rstd, nw, ch * 32);
    if (dst) pro_store32(dst + ch * 32, x);
  }
}

}  // namespace lb
