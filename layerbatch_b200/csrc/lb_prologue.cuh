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
                                                int tok0, int n, int h, int lane) {
  ProRow r;
  r.n = n;
  r.h = h;
  r.x = make_uint4(0, 0, 0, 0);
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  const long long t = (long long)tok0 + n;
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

// Normalise, rotate and store one loaded row (value rows are stored as they are).  All 32
// lanes of the warp call it together (warp shuffles), also for rows with h = -1.
__device__ __forceinline__ void prologue_store(const LbPrologueArgs& a, const ProStage* st,
                                               int tok0, const ProRow& r, int lane,
                                               const uint4& qw, const uint4& kw) {
  const int Hq = (int)a.num_q_heads, Hkv = (int)a.num_kv_heads;
  if (r.h >= Hq + Hkv) {   // value row (a warp-uniform branch: the row is the warp's)
    const long long row = (long long)st->slot[r.n] * Hkv * PRO_D + (long long)(r.h - Hq - Hkv) * PRO_D;
    reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.v_cache) + row)[lane] = r.x;
    return;
  }
  const bool is_q = r.h < Hq;
  float x[8] = {bf16_lo(r.x.x), bf16_hi(r.x.x), bf16_lo(r.x.y), bf16_hi(r.x.y),
                bf16_lo(r.x.z), bf16_hi(r.x.z), bf16_lo(r.x.w), bf16_hi(r.x.w)};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float rstd = 1.0f / sqrtf(__fadd_rn(ss / (float)PRO_D, a.eps));
  const uint4 wr = is_q ? qw : kw;
  const float w[8] = {bf16_lo(wr.x), bf16_hi(wr.x), bf16_lo(wr.y), bf16_hi(wr.y),
                      bf16_lo(wr.z), bf16_hi(wr.z), bf16_lo(wr.w), bf16_hi(wr.w)};
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    y[i] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[i], rstd), __fadd_rn(1.0f, w[i]))));
  // partial RoPE: dims [0, rot/2) pair with [rot/2, rot); lanes < rot/16 hold the first
  // half, the next rot/16 lanes the second
  const int rot = (int)a.rotary_dim;
  const int hl = rot / 16;
  const bool first = lane < hl, second = lane >= hl && lane < 2 * hl;
  const int partner = first ? lane + hl : (second ? lane - hl : lane);
  float pv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) pv[i] = __shfl_sync(0xffffffffu, y[i], partner);
  if (r.h < 0) return;
  if (first || second) {
    const float* cs = st->cs[r.n];
    const int f0 = (first ? lane : lane - hl) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = cs[f0 + i], sn = cs[rot / 2 + f0 + i];
      const float t = first ? __fsub_rn(__fmul_rn(y[i], c), __fmul_rn(pv[i], sn))   // x1 c - x2 s
                            : __fadd_rn(__fmul_rn(y[i], c), __fmul_rn(pv[i], sn));  // x2 c + x1 s
      y[i] = __bfloat162float(__float2bfloat16_rn(t));
    }
  }
  const uint4 outv = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  const long long t = (long long)tok0 + r.n;
  if (is_q) {
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.q_out) + t * a.q_out_stride_tok +
                         (long long)r.h * a.q_out_stride_head;
    reinterpret_cast<uint4*>(dst)[lane] = outv;
  } else {
    const long long row = (long long)st->slot[r.n] * Hkv * PRO_D + (long long)(r.h - Hq) * PRO_D;
    reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.k_cache) + row)[lane] = outv;
  }
}

// One task: tokens [tok0, tok0 + ntok), ntok <= PRO_TASK_TOKENS.  Every thread of the block
// calls it (it stages with the whole block and meets at __syncthreads); `nwarps` warps
// (warp ids [0, nwarps)) take the rows.  The caller separates consecutive tasks with a
// __syncthreads, as the staging area is reused.
__device__ __forceinline__ void prologue_task(const LbPrologueArgs& a, int tok0, int ntok,
                                              ProStage* st, int warp, int nwarps, int lane,
                                              int* status) {
  const int rot = (int)a.rotary_dim;
  for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
    const long long s = (long long)a.slot_mapping[tok0 + i];
    if (s >= a.num_slots) report(status, LB_DEV_BAD_INDEX);
    st->slot[i] = (s < 0 || s >= a.num_slots) ? -1 : (int)s;
  }
  for (int e = threadIdx.x; e < ntok * rot; e += blockDim.x) {
    const int i = e / rot, c = e - (e / rot) * rot;
    long long pos = a.positions[tok0 + i];
    if (pos < 0 || pos >= a.max_position) {
      if (c == 0) report(status, LB_DEV_BAD_INDEX);
      pos = pos < 0 ? 0 : a.max_position - 1;
    }
    st->cs[i][c] = a.cos_sin_cache[pos * rot + c];
  }
  __syncthreads();
  if (warp >= nwarps) return;
  const uint4 qw = reinterpret_cast<const uint4*>(a.q_norm_w)[lane];
  const uint4 kw = reinterpret_cast<const uint4*>(a.k_norm_w)[lane];
  const int nh = (int)(a.num_q_heads + 2 * a.num_kv_heads);
  const int rows = ntok * nh;
  for (int j0 = warp * PRO_BATCH; j0 < rows; j0 += nwarps * PRO_BATCH) {
    ProRow r[PRO_BATCH];
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) {
      const int j = j0 + i;
      if (j < rows) {
        r[i] = prologue_load(a, st, tok0, j / nh, j - (j / nh) * nh, lane);
      } else {
        r[i].h = -1;
        r[i].n = 0;
        r[i].x = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int i = 0; i < PRO_BATCH; ++i) prologue_store(a, st, tok0, r[i], lane, qw, kw);
  }
}

}  // namespace lb
