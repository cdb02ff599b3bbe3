// POD attention for sm_100a: one persistent launch that runs causal prefill tiles and
// split-KV decode items over a paged KV cache, side by side on different SMs.
//
// Work items come from two device-built queues (k_pod_plan).  A CTA starts in the mode
// the host assigned to it (prefill for blockIdx < n_prefill_ctas, decode otherwise),
// drains that queue, then switches once to the other queue, so prefill (tensor-bound)
// and decode (HBM-bound) items overlap across SMs and the tail is balanced.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + tcgen05.mma issuer,
// warps 2..9 = softmax / epilogue: two warpgroups, one thread per TMEM lane each.  Decode
// items use warpgroup 0 only; prefill items split every score row between the two
// warpgroups (32 keys each) and each warpgroup owns half of the O columns.
//
// KV tiles are 128 tokens x 256 dims, loaded by TMA as four 64-dim chunks of
// [128 rows x 128 B] (128B swizzle), the same layout for K and V.  A 128-token tile never
// crosses a 256-token page, so one page-table lookup addresses a whole tile.
//
// Decode item (b, kv_head, split): S^T = K . Q^T (M = 128 tokens, N = 16 q-heads of the
// GQA group, K = 256) and O^T = V^T . P^T (M = 128 dims x 2, N = 16, K = 128 tokens,
// V^T read MN-major straight from the V tile).  Online softmax keeps per-head state in
// the 128 softmax threads; partial O and the log2-sum-exp of each split go to the
// workspace and k_pod_merge combines them.
// Prefill item (b, q_head, q_tile): S = Q . K^T (M = 128 queries, N = 64 keys) and
// O += P . V (N = 256 dims, V MN-major, P bf16 read from TMEM as the A operand), O
// accumulating in TMEM with per-row rescaling;
// bottom-right causal mask; the epilogue applies sigmoid(gate) and writes bf16 rows of
// the o_proj input.
#pragma once

#include <cuda.h>
#include "lb_common.cuh"
#include "lb_prologue.cuh"

namespace lb {

constexpr int POD_THREADS = 320;
constexpr int POD_KV = 128;          // tokens per K or V tile
constexpr int POD_D = 256;           // head_dim
constexpr int POD_CHUNK = POD_KV * 128;          // 16 KB: one 64-dim chunk of a tile
constexpr int POD_TILE = 4 * POD_CHUNK;          // 64 KB
constexpr int POD_QD_BYTES = 16 * POD_D * 2;     // 8 KB decode Q (16 head rows)
constexpr int POD_PD_BYTES = 16 * POD_KV * 2;    // 4 KB decode P^T
constexpr int POD_QP_BYTES = POD_KV * POD_D * 2; // 64 KB prefill Q
constexpr int POD_PP_BYTES = POD_KV * POD_KV * 2;// 32 KB prefill P
constexpr int POD_DATA = 224 * 1024;
constexpr int POD_MISC = 2048;
constexpr int POD_SMEM = 1024 + POD_DATA + POD_MISC;
constexpr int POD_TMEM_COLS = 512;
constexpr int DEC_SLOTS = 3;
// prefill: 64-key K/V tiles (32 KB) in separate K and V rings, K two tiles deep, V three
// (with the MMAs issued as their inputs arrive, the scores run ahead and PV_j, which also
// waits for the softmax, holds its V slot longest); P goes to TMEM, not shared memory
constexpr int PF_KV = 64;
constexpr int PF_CHUNK = PF_KV * 128;            // 8 KB: one 64-dim chunk of a prefill tile
constexpr int PF_TILE = 4 * PF_CHUNK;            // 32 KB
constexpr int PF_KSLOTS = 2;                     // K ring: barriers kv_*[0, 2)
constexpr int PF_VSLOTS = 3;                     // V ring: barriers kv_*[2, 5)
// prefill shared-memory map: [K ring 2 x 32 KB][V ring 3 x 32 KB][Q 64 KB]
constexpr int PF_K_OFF = 0;
constexpr int PF_V_OFF = PF_KSLOTS * PF_TILE;
constexpr int PF_Q_OFF = PF_V_OFF + PF_VSLOTS * PF_TILE;
static_assert(PF_Q_OFF + POD_QP_BYTES <= POD_DATA, "prefill shared-memory map exceeds the data region");
// prefill TMEM map: S double buffer [0, 128) (fp32 128 x 64 each), bf16 P double buffer
// [PF_P_COL, PF_P_COL + 64) (128 x 64 keys, two keys per 32-bit column, the A operand of
// the PV MMA read from TMEM), O [256, 512)
constexpr int PF_P_COL = 128;
// decode shared-memory map: [ring 3 x 64 KB][Q x2][P^T x2]
static_assert(DEC_SLOTS * POD_TILE + 2 * POD_QD_BYTES + 2 * POD_PD_BYTES <= POD_DATA,
              "decode shared-memory map exceeds the data region");

struct PodParams {
  int* status;
  const int4* pf_items;
  const int* pf_count;
  int* pf_next;
  const int4* dec_items;
  const int* dec_count;
  int* dec_next;
  const int32_t* block_tables;
  long long bt_stride;
  const int32_t* context_lens;
  const int32_t* cu_seqlens_q;
  const __nv_bfloat16* gate;   // output gate (pre-sigmoid) or null for no gate
  long long gate_st, gate_sh;
  __nv_bfloat16* ogated;       // [N, Hq*D] gated attention output (o_proj input) or null
  __nv_bfloat16* attn_out;     // optional [N, Hq*D] pre-gate attention output
  float* part_o;               // [B, max_splits, Hq, D]
  float* part_lse;             // [B, max_splits, Hq]
  int max_splits;
  int Hq, Hkv, gqa;
  int page_size, num_pages;
  int split_tokens;
  int n_prefill_ctas;
  int qd_bytes;                // bytes of one decode Q tile (4 chunks x rows x 128 B)
  float scale_log2;
  // Fused prologue (optional, pro_tasks = 0: off).  Before attention, the CTAs take tasks
  // of PRO_TASK_TOKENS tokens from pro_next and run the prologue of their rows (query to
  // `q`, key / value into the cache); seq_ready[b] then counts sequence b's new tokens
  // done (release).  An item's producer waits for its sequence's count to reach what the
  // item reads before it loads Q / K / V.  Every CTA finishes claiming tasks before it
  // starts any item, so a wait only ever waits for tasks running on resident CTAs.
  LbPrologueArgs pro;
  int pro_tasks;
  int* pro_next;
  int* pro_done;        // tasks finished (release); == pro_tasks: every row is stored
  int* seq_ready;
  int num_tokens;
  int num_seqs;
};



struct PodBars {
  uint64_t kv_full[5], kv_empty[5];
  uint64_t item_full[2], item_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], o_full[2];
  uint64_t q_empty;
  uint64_t drain;
  int4 items[2];
  uint32_t tmem_base;
  int abort;
  float red[2][4][16];
  float lred[4][16];
  float psum[2][128];      // prefill: per-warpgroup partial row sums at the end of an item
  int pro_task;            // fused prologue: the task the CTA works on
  int skip_pass;           // the second pass's queue was already empty
};

static_assert(sizeof(PodBars) <= POD_MISC, "PodBars exceeds the reserved shared memory");

struct PodCounters {  // per-role running positions, kept across items and modes
  uint32_t kv, item, s, o, qp, kv2;  // kv2: prefill V tiles (K tiles use kv)
};

// Sequence of packed token `tok`: the last b with cu_seqlens_q[b] <= tok.
__device__ __forceinline__ int seq_of_token(const PodParams& p, int tok) {
  int lo = 0, hi = p.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cu_seqlens_q[mid] <= tok) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Bounded wait until sequence b has `need` new tokens through the fused prologue; then
// its query rows and stored K/V rows may be loaded by TMA by this thread.  `all_ready` is
// the thread's own note that every task was seen finished (after which there is nothing
// to wait for and the fences below have been run once).  No-op without the prologue.
__device__ __forceinline__ bool wait_seq_ready(const PodParams& p, int b, int need,
                                               bool& all_ready) {
  if (p.pro_tasks == 0 || all_ready) return true;
  if (ld_acquire_gpu(p.pro_done) >= p.pro_tasks) {
    fence_proxy_async_global();
    all_ready = true;
    return true;
  }
  if (ld_acquire_gpu(p.seq_ready + b) < need) {
    const long long t0 = clock64();
    while (ld_acquire_gpu(p.seq_ready + b) < need) {
      if (clock64() - t0 > (long long)LB_SPIN_LIMIT_CYCLES) {
        report(p.status, LB_DEV_TIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
  fence_proxy_async_global();
  return true;
}

// The fused prologue phase, run by every CTA before its first attention item: the CTA's
// warps take tasks of PRO_TASK_TOKENS consecutive tokens from the counter until every task
// is claimed (rows straight from global memory, prologue_rows_direct).  A CTA thus starts
// items only once every task has been claimed by a running CTA, and an item's wait for its
// sequence's rows only ever waits for tasks in progress.
__device__ __forceinline__ void pod_prologue_phase(const PodParams& p, PodBars* bars) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const ProNorm nw = prologue_norm(p.pro, lane);
  while (true) {
    if (threadIdx.x == 0) bars->pro_task = atomicAdd(p.pro_next, 1);
    __syncthreads();
    const int t = bars->pro_task;
    if (t >= p.pro_tasks) break;
    const int t0 = t * PRO_TASK_TOKENS;
    const int ntok = min(PRO_TASK_TOKENS, p.num_tokens - t0);
    prologue_rows_direct(p.pro, t0, ntok, warp, POD_THREADS / 32, lane, nw, p.status);
    // the rows are read back by TMA (async proxy) on other SMs
    fence_proxy_async_global();
    __threadfence();
    __syncthreads();
    if ((int)threadIdx.x < ntok) red_release_gpu_add(p.seq_ready + seq_of_token(p, t0 + threadIdx.x), 1);
    if (threadIdx.x == 0) red_release_gpu_add(p.pro_done, 1);
  }
}

__device__ __forceinline__ int kv_page_row(const PodParams& p, int b, int tok) {
  const int pi = tok / p.page_size;
  int blk = p.block_tables[(long long)b * p.bt_stride + pi];
  if (blk < 0 || blk >= p.num_pages) {
    report(p.status, LB_DEV_BAD_INDEX);
    blk = 0;
  }
  return blk * p.page_size + (tok - pi * p.page_size);
}

// Load a 128-token K or V tile (4 chunks) for kv head `kvh` starting at token `tok`.
__device__ __forceinline__ void load_kv_tile(uint8_t* dst, const CUtensorMap* map,
                                             uint64_t* bar, int kvh, int row) {
#pragma unroll
  for (int c = 0; c < 4; ++c) tma_load_3d(dst + c * POD_CHUNK, map, bar, c * 64, kvh, row);
}

// Decode ring order of one item of n tiles: the first DEC_KAHEAD K tiles, then V0, K(A),
// V1, K(A+1), ..., then the remaining V tiles (A = DEC_KAHEAD; with A = 2: K0, K1, V0, K2,
// V1, ..., K(n-1), V(n-2), V(n-1)).  K runs ahead of V, so the K tile of the next S MMA is
// never queued behind a V tile that waits for the current softmax, and each V tile streams
// in while its scores are being turned into P.
#ifndef LB_DEC_KAHEAD
#define LB_DEC_KAHEAD 2
#endif
constexpr int DEC_KAHEAD = LB_DEC_KAHEAD;
// With DEC_SLOTS = 3 and the MMA order S_j, PV_{j-1}: V_j takes the slot of the load three
// positions earlier, which for DEC_KAHEAD = 4 is K_{j+2}, freed only by S_{j+2}, issued
// after PV_j: a deadlock.  1 to 3 are safe (2 measured fastest).
static_assert(DEC_KAHEAD >= 1 && DEC_KAHEAD <= 3, "decode ring order");
__device__ __forceinline__ int dec_pos_k(int j) {
  return j < DEC_KAHEAD ? j : DEC_KAHEAD + 2 * (j - DEC_KAHEAD) + 1;
}
__device__ __forceinline__ int dec_pos_v(int j, int n) {
  const int a = min(n, DEC_KAHEAD), m = max(0, n - DEC_KAHEAD);
  return j < m ? DEC_KAHEAD + 2 * j : a + 2 * m + (j - m);
}
// Ring position q of an item of n tiles -> its tile, and whether it is the V tile (the
// inverse of dec_pos_k / dec_pos_v).
__device__ __forceinline__ int dec_ring_tile(int q, int n, bool& is_v) {
  const int a = min(n, DEC_KAHEAD), m = max(0, n - DEC_KAHEAD);
  if (q < a) {
    is_v = false;
    return q;
  }
  if (q < a + 2 * m) {
    const int r = q - a;
    is_v = !(r & 1);
    return is_v ? (r >> 1) : (r >> 1) + DEC_KAHEAD;
  }
  is_v = true;
  return m + (q - a - 2 * m);
}

// Decode TMEM columns: S^T [2 buffers][4 chunk partials][16 heads], O^T [2 buffers][2 dim
// halves][4 token-quarter partials][16 heads].
constexpr int DEC_S_COL = 0;
constexpr int DEC_O_COL = 128;

// 32 lanes x 32 bit, N (8 or 16) consecutive TMEM columns per thread.
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 8 || N == 16, "8 or 16 columns");
  if constexpr (N == 8) tmem_ld8(taddr, r); else tmem_ld16(taddr, r);
}

// Sum of the four token-quarter partials of each dim half of a decode O^T buffer (the
// first NH of the 16 head columns of each partial).
template <int NH>
__device__ __forceinline__ void dec_load_o(uint32_t taddr, uint32_t (&o0)[NH], uint32_t (&o1)[NH]) {
  uint32_t a[NH], b[NH], c[NH];
  tmem_ldn<NH>(taddr, o0);
  tmem_ldn<NH>(taddr + 16, a);
  tmem_ldn<NH>(taddr + 32, b);
  tmem_ldn<NH>(taddr + 48, c);
  tmem_wait_ld();
#pragma unroll
  for (int h = 0; h < NH; ++h)
    o0[h] = __float_as_uint((__uint_as_float(o0[h]) + __uint_as_float(a[h])) +
                            (__uint_as_float(b[h]) + __uint_as_float(c[h])));
  tmem_ldn<NH>(taddr + 64, o1);
  tmem_ldn<NH>(taddr + 80, a);
  tmem_ldn<NH>(taddr + 96, b);
  tmem_ldn<NH>(taddr + 112, c);
  tmem_wait_ld();
#pragma unroll
  for (int h = 0; h < NH; ++h)
    o1[h] = __float_as_uint((__uint_as_float(o1[h]) + __uint_as_float(a[h])) +
                            (__uint_as_float(b[h]) + __uint_as_float(c[h])));
}

// Byte offset of element (r, c) in a K-major SW128 tile of 64-element (128 B) rows.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + ((c & 7) << 1));
}

// One decode item of the softmax warpgroup (128 threads, thread = token row of each
// 128-token tile): online softmax over the item's tiles for the NH head columns of the
// S / O^T accumulators, P^T to shared memory for the PV MMA, and the split's partial O and
// log2-sum-exp.  NH = 8 serves GQA groups of up to 8 heads with half the registers,
// TMEM loads and instructions of NH = 16; the MMAs still compute 16 head columns, and
// columns NH..15 of S and O^T (whatever their contents) are never read, since a column of
// an MMA result depends only on the same column of its B operand.  Returns false when the
// item must be abandoned (a wait gave up); `ok` is false then.
template <int NH>
__device__ __forceinline__ bool dec_softmax_item(const PodParams& p, PodBars* bars, PodCounters& cnt,
                                                 uint8_t* smem, uint8_t* kv_base, int nslots,
                                                 uint32_t tl, int quad, int lane, int row, int tid,
                                                 int b, int ctx, int kvh, int split, bool& ok) {
  const int t_begin = split * p.split_tokens;
  const int t_end = min(ctx, t_begin + p.split_tokens);
  const int ntiles = (t_end - t_begin + POD_KV - 1) / POD_KV;
  const uint32_t kvbase = cnt.kv;
  cnt.kv += 2 * ntiles;
  float m[NH], l[NH], a0[NH], a1[NH], ap[NH];
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
    a0[h] = 0.f;
    a1[h] = 0.f;
    ap[h] = 1.f;
  }
  for (int j = 0; j <= ntiles; ++j) {
    if (j < ntiles) {
      const int sb = cnt.s & 1;
      // a failed wait (here or earlier in the item) is agreed on at this tile's
      // barrier below, where all 128 threads leave the item together
      if (ok) ok = mbar_wait_warp(&bars->s_full[sb], (cnt.s >> 1) & 1, p.status);
      tc_fence_after();
      uint32_t r[NH];
      {
        uint32_t r1[NH], r2[NH], r3[NH];
        tmem_ldn<NH>(tl + DEC_S_COL + sb * 64, r);
        tmem_ldn<NH>(tl + DEC_S_COL + sb * 64 + 16, r1);
        tmem_ldn<NH>(tl + DEC_S_COL + sb * 64 + 32, r2);
        tmem_ldn<NH>(tl + DEC_S_COL + sb * 64 + 48, r3);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < NH; ++h)
          r[h] = __float_as_uint((__uint_as_float(r[h]) + __uint_as_float(r1[h])) +
                                 (__uint_as_float(r2[h]) + __uint_as_float(r3[h])));
      }
      tc_fence_before();
      mbar_arrive(&bars->s_empty[sb]);
      ++cnt.s;
      const bool valid = t_begin + j * POD_KV + row < t_end;
      float s[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h)
        s[h] = (valid && h < p.gqa) ? __uint_as_float(r[h]) * p.scale_log2 : -INFINITY;
      // tile max per head across the 128 token rows
      const int par = j & 1;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        float v = s[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) bars->red[par][quad][h] = v;
      }
      if (named_bar_any(1, 128, !ok)) { ok = false; break; }
      const int ob = cnt.o & 1;
      const uint32_t pt = smem_u32(smem + DEC_SLOTS * POD_TILE + 2 * POD_QD_BYTES +
                                   ob * POD_PD_BYTES);
      float al[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float mt = fmaxf(fmaxf(bars->red[par][0][h], bars->red[par][1][h]),
                               fmaxf(bars->red[par][2][h], bars->red[par][3][h]));
        const float mn = fmaxf(m[h], mt);
        al[h] = (m[h] == -INFINITY) ? 1.f : exp2_approx(m[h] - mn);
        const float e = (mn == -INFINITY) ? 0.f : exp2_approx(s[h] - mn);
        l[h] = l[h] * al[h] + e;
        m[h] = mn;
        // P^T[h][token]: K-major rows of 128 tokens, two 64-token chunks
        st_shared_u16(pt + (row >> 6) * 2048 + sw128_off(h, row & 63),
                      __bfloat16_as_ushort(__float2bfloat16_rn(e)));
      }
      // tokens past the end of the last tile: zero their V rows (stale cache bytes
      // could be NaN, and 0 * NaN would poison O^T)
      if (t_begin + (j + 1) * POD_KV > t_end) {
        const uint32_t vp = kvbase + dec_pos_v(j, ntiles);
        if (!mbar_wait_warp(&bars->kv_full[vp % nslots], (vp / nslots) & 1, p.status)) {
          ok = false;
        } else if (!valid) {
          const uint32_t v = smem_u32(kv_base + (vp % nslots) * POD_TILE) + row * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int u = 0; u < 8; ++u) st_shared_v4(v + c * POD_CHUNK + u * 16, 0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[ob]);
      if (j > 0 && ok) {
        // accumulate O_{j-1} (scale of tile j-1), deferred behind P_j
        const int pb = ob ^ 1;
        ok = mbar_wait_warp(&bars->o_full[pb], ((cnt.o - 1) >> 1) & 1, p.status);
        if (ok) {
          tc_fence_after();
          uint32_t o0[NH], o1[NH];
          dec_load_o<NH>(tl + DEC_O_COL + pb * 128, o0, o1);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            a0[h] = a0[h] * ap[h] + __uint_as_float(o0[h]);
            a1[h] = a1[h] * ap[h] + __uint_as_float(o1[h]);
          }
          tc_fence_before();
        }
      }
#pragma unroll
      for (int h = 0; h < NH; ++h) ap[h] = al[h];
      ++cnt.o;
    } else {
      // final O
      const int pb = (cnt.o - 1) & 1;
      if (ok) ok = mbar_wait_warp(&bars->o_full[pb], ((cnt.o - 1) >> 1) & 1, p.status);
      if (ok) {
        tc_fence_after();
        uint32_t o0[NH], o1[NH];
        dec_load_o<NH>(tl + DEC_O_COL + pb * 128, o0, o1);
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          a0[h] = a0[h] * ap[h] + __uint_as_float(o0[h]);
          a1[h] = a1[h] * ap[h] + __uint_as_float(o1[h]);
        }
        tc_fence_before();
      }
    }
  }
  // row sums across the 128 threads
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    float v = l[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) bars->lred[quad][h] = v;
  }
  if (named_bar_any(1, 128, !ok)) return false;
  const long long pbase = ((long long)b * p.max_splits + split) * p.Hq;
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    if (h < p.gqa) {
      const float ls = bars->lred[0][h] + bars->lred[1][h] + bars->lred[2][h] + bars->lred[3][h];
      const float inv = ls > 0.f ? 1.f / ls : 0.f;
      const int hq = kvh * p.gqa + h;
      float* dst = p.part_o + (pbase + hq) * POD_D;
      dst[row] = a0[h] * inv;
      dst[row + 128] = a1[h] * inv;
      if (tid == h) p.part_lse[pbase + hq] = m[h] + log2f(ls);
    }
  }
  return true;
}

__global__ void __launch_bounds__(POD_THREADS, 1)
    k_pod_attn(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
               const __grid_constant__ CUtensorMap tmK64, const __grid_constant__ CUtensorMap tmV64,
               const __grid_constant__ CUtensorMap tmQd, const __grid_constant__ CUtensorMap tmQp,
               const PodParams p) {
  pdl_entry();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  PodBars* bars = reinterpret_cast<PodBars*>(smem + POD_DATA);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  volatile int* abortp = &bars->abort;

  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, POD_TMEM_COLS);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) bars->abort = 0;
  PodCounters cnt = {0, 0, 0, 0, 0, 0};
  if (p.pro_tasks > 0) pod_prologue_phase(p, bars);
  bool pro_all_ready = false;   // producer lanes: every prologue task seen finished

  const bool pf_first = (int)blockIdx.x < p.n_prefill_ctas;
  for (int pass = 0; pass < 2; ++pass) {
    const bool prefill = (pass == 0) ? pf_first : !pf_first;
    const int nslots = DEC_SLOTS;   // decode ring (prefill: the PF_KSLOTS / PF_VSLOTS rings)

    if (threadIdx.x == 0) {
      for (int i = 0; i < 5; ++i) {
        mbar_init(&bars->kv_full[i], 1);
        mbar_init(&bars->kv_empty[i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&bars->item_full[i], 1);
        mbar_init(&bars->item_empty[i], 1);
        mbar_init(&bars->s_full[i], 1);
        mbar_init(&bars->s_empty[i], prefill ? 256 : 128);
        mbar_init(&bars->p_full[i], prefill ? 256 : 128);
        mbar_init(&bars->o_full[i], 1);
      }
      mbar_init(&bars->q_empty, 1);
      mbar_init(&bars->drain, 1);
      fence_barrier_init();
    }
    cnt = {0, 0, 0, 0, 0, 0};
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    uint8_t* kv_base = smem;  // ring of `nslots` 64 KB tiles

    if (warp == 0) {
      // ============================================================ producer
      // lane 0: items, Q, decode K/V tiles, prefill K tiles; lane 1: prefill V tiles, so
      // K tiles never wait behind a V tile whose ring slot is still in use
      if (lane == 0) {
        const int4* items = prefill ? p.pf_items : p.dec_items;
        const int n_items = *(prefill ? p.pf_count : p.dec_count);
        int* next = prefill ? p.pf_next : p.dec_next;
        while (!*abortp) {
          const int islot = cnt.item & 1;
          const uint32_t iph = (cnt.item >> 1) & 1;
          if (!mbar_wait(&bars->item_empty[islot], iph ^ 1, p.status)) { *abortp = 1; break; }
          const int idx = atomicAdd(next, 1);
          if (idx >= n_items) {
            bars->items[islot] = make_int4(-1, 0, 0, 0);
            mbar_arrive(&bars->item_full[islot]);
            ++cnt.item;
            break;
          }
          const int4 it = items[idx];
          {
            // fused prologue: the item's query rows and new K/V rows must be stored
            const int bq = it.x;
            const int need = prefill ? p.cu_seqlens_q[bq + 1] - p.cu_seqlens_q[bq] : 1;
            if (!wait_seq_ready(p, bq, need, pro_all_ready)) {
              *abortp = 1;
              bars->items[islot] = make_int4(-1, 0, 0, 0);
              mbar_arrive(&bars->item_full[islot]);
              ++cnt.item;
              break;
            }
          }
          bars->items[islot] = it;
          const int b = it.x;
          const int ctx = p.context_lens[b];
          int kvh, t_begin, ntiles;
          if (prefill) {
            const int qlen = p.cu_seqlens_q[b + 1] - p.cu_seqlens_q[b];
            const int h = it.y, qt = it.z;
            kvh = h / p.gqa;
            const int kv_end = min(ctx, ctx - qlen + (qt + 1) * POD_KV);
            t_begin = 0;
            ntiles = (kv_end + PF_KV - 1) / PF_KV;
            // the single prefill Q buffer is free once the previous item's S MMAs finish
            if (!mbar_wait(&bars->q_empty, (cnt.qp & 1) ^ 1, p.status)) { *abortp = 1; break; }
            ++cnt.qp;
            uint8_t* qbuf = smem + PF_Q_OFF;
            const int row0 = p.cu_seqlens_q[b] + qt * POD_KV;
            mbar_arrive_expect_tx(&bars->item_full[islot], POD_QP_BYTES);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_3d(qbuf + c * POD_CHUNK, &tmQp, &bars->item_full[islot], c * 64, h, row0);
          } else {
            kvh = it.y;
            const int split = it.z;
            t_begin = split * p.split_tokens;
            const int t_end = min(ctx, t_begin + p.split_tokens);
            ntiles = (t_end - t_begin + POD_KV - 1) / POD_KV;
            uint8_t* qbuf = smem + DEC_SLOTS * POD_TILE + islot * POD_QD_BYTES;
            const int tok = p.cu_seqlens_q[b];
            mbar_arrive_expect_tx(&bars->item_full[islot], p.qd_bytes);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_3d(qbuf + c * 2048, &tmQd, &bars->item_full[islot], c * 64,
                          kvh * p.gqa, tok);
          }
          ++cnt.item;
          if (prefill) {
            for (int j = 0; j < ntiles && !*abortp; ++j) {
              const int slot = cnt.kv % PF_KSLOTS;
              if (!mbar_wait(&bars->kv_empty[slot], ((cnt.kv / PF_KSLOTS) & 1) ^ 1, p.status)) { *abortp = 1; break; }
              const int row = kv_page_row(p, b, j * PF_KV);
              mbar_arrive_expect_tx(&bars->kv_full[slot], PF_TILE);
              uint8_t* dst = smem + PF_K_OFF + slot * PF_TILE;
#pragma unroll
              for (int c = 0; c < 4; ++c)
                tma_load_3d(dst + c * PF_CHUNK, &tmK64, &bars->kv_full[slot], c * 64, kvh, row);
              ++cnt.kv;
            }
          } else {
            for (int j = 0; j < 2 * ntiles && !*abortp; ++j) {
              const int slot = cnt.kv % nslots;
              const uint32_t ph = (cnt.kv / nslots) & 1;
              if (!mbar_wait(&bars->kv_empty[slot], ph ^ 1, p.status)) { *abortp = 1; break; }
              bool is_v;
              const int tile = dec_ring_tile(j, ntiles, is_v);
              const int row = kv_page_row(p, b, t_begin + tile * POD_KV);
              mbar_arrive_expect_tx(&bars->kv_full[slot], POD_TILE);
              load_kv_tile(kv_base + slot * POD_TILE, is_v ? &tmV : &tmK, &bars->kv_full[slot],
                           kvh, row);
              ++cnt.kv;
            }
          }
        }
      } else if (lane == 1 && prefill) {
        // V loader: follows the item sequence through item_full
        while (!*abortp) {
          const int islot = cnt.item & 1;
          if (!mbar_wait(&bars->item_full[islot], (cnt.item >> 1) & 1, p.status)) { *abortp = 1; break; }
          const int4 it = bars->items[islot];
          ++cnt.item;
          if (it.x < 0) break;
          const int b = it.x;
          const int ctx = p.context_lens[b];
          const int qlen = p.cu_seqlens_q[b + 1] - p.cu_seqlens_q[b];
          // lane 0 saw the count before publishing the item; this lane's own acquire
          // orders its V loads after the prologue's stores
          if (!wait_seq_ready(p, b, qlen, pro_all_ready)) { *abortp = 1; break; }
          const int kvh = it.y / p.gqa;
          const int kv_end = min(ctx, ctx - qlen + (it.z + 1) * POD_KV);
          const int ntiles = (kv_end + PF_KV - 1) / PF_KV;
          for (int j = 0; j < ntiles && !*abortp; ++j) {
            const int slot = cnt.kv2 % PF_VSLOTS;
            if (!mbar_wait(&bars->kv_empty[PF_KSLOTS + slot], ((cnt.kv2 / PF_VSLOTS) & 1) ^ 1, p.status)) { *abortp = 1; break; }
            const int row = kv_page_row(p, b, j * PF_KV);
            mbar_arrive_expect_tx(&bars->kv_full[PF_KSLOTS + slot], PF_TILE);
            uint8_t* dst = smem + PF_V_OFF + slot * PF_TILE;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_3d(dst + c * PF_CHUNK, &tmV64, &bars->kv_full[PF_KSLOTS + slot], c * 64, kvh, row);
            ++cnt.kv2;
          }
        }
      }
    } else if (warp == 1) {
      // ============================================================ MMA issuer
      if (elect_one_sync()) {
        const uint32_t idesc_s = prefill ? umma_idesc_bf16(128, PF_KV, false, false)
                                         : umma_idesc_bf16(128, 16, false, false);
        const uint32_t idesc_o = prefill ? umma_idesc_bf16(128, 256, false, true)
                                         : umma_idesc_bf16(128, 16, true, false);
        while (!*abortp) {
          const int islot = cnt.item & 1;
          const uint32_t iph = (cnt.item >> 1) & 1;
          if (!mbar_wait(&bars->item_full[islot], iph, p.status)) { *abortp = 1; break; }
          const int4 it = bars->items[islot];
          ++cnt.item;
          if (it.x < 0) break;
          const int b = it.x;
          const int ctx = p.context_lens[b];
          int ntiles;
          if (prefill) {
            const int qlen = p.cu_seqlens_q[b + 1] - p.cu_seqlens_q[b];
            const int kv_end = min(ctx, ctx - qlen + (it.z + 1) * POD_KV);
            ntiles = (kv_end + PF_KV - 1) / PF_KV;
          } else {
            const int t_begin = it.z * p.split_tokens;
            const int t_end = min(ctx, t_begin + p.split_tokens);
            ntiles = (t_end - t_begin + POD_KV - 1) / POD_KV;
          }
          const uint32_t base = cnt.kv, vbase = cnt.kv2;
          const uint32_t qaddr = prefill ? smem_u32(smem + PF_Q_OFF)
                                         : smem_u32(smem + DEC_SLOTS * POD_TILE + islot * POD_QD_BYTES);
          bool ok = true;
          if (prefill) {
            // S and PV MMAs are issued each as soon as its own inputs are ready (polled, not
            // waited on in a fixed order): S_{j+2} needs only the softmax to have read S_j
            // (and K_{j+2}), PV_j needs P_j (and V_j).  A fixed S, PV, S, PV order would hold
            // the next scores behind the softmax -> PV hand-off of an earlier tile.  Bounded:
            // the spin limit counts from the last MMA issued.
            int ns = 0, npv = 0;
            unsigned long long t_last = clock64();
            while (npv < ntiles) {
              bool moved = false;
              if (ns < ntiles) {
                const uint32_t kp = base + ns;
                const int ks = kp % PF_KSLOTS;
                const int sb = cnt.s & 1;
                if (mbar_try_wait(&bars->s_empty[sb], ((cnt.s >> 1) & 1) ^ 1) &&
                    mbar_try_wait(&bars->kv_full[ks], (kp / PF_KSLOTS) & 1)) {
                  tc_fence_after();
                  const uint32_t kaddr = smem_u32(smem + PF_K_OFF + ks * PF_TILE);
                  const uint32_t d = tmem + sb * PF_KV;
#pragma unroll
                  for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                      umma_bf16(d, umma_desc_sw128(qaddr + c * POD_CHUNK + kk * 32, 16, 1024),
                                umma_desc_sw128(kaddr + c * PF_CHUNK + kk * 32, 16, 1024), idesc_s,
                                (c | kk) != 0);
                  umma_commit(&bars->s_full[sb]);
                  umma_commit(&bars->kv_empty[ks]);
                  if (ns == ntiles - 1) umma_commit(&bars->q_empty);
                  ++cnt.s;
                  ++ns;
                  moved = true;
                }
              }
              if (npv < ns) {
                const uint32_t vp = vbase + npv;
                const int vs = PF_KSLOTS + (int)(vp % PF_VSLOTS);
                const int ob = cnt.o & 1;
                if (mbar_try_wait(&bars->p_full[ob], (cnt.o >> 1) & 1) &&
                    mbar_try_wait(&bars->kv_full[vs], (vp / PF_VSLOTS) & 1)) {
                  tc_fence_after();
                  const uint32_t vaddr = smem_u32(smem + PF_V_OFF + (vp % PF_VSLOTS) * PF_TILE);
                  // A = P from TMEM: 16 keys (8 columns) per MMA
                  const uint32_t pcol = tmem + PF_P_COL + ob * (PF_KV / 2);
                  const uint32_t d = tmem + 256;
#pragma unroll
                  for (int kk = 0; kk < PF_KV / 16; ++kk)
                    umma_bf16_ts(d, pcol + kk * 8,
                                 umma_desc_sw128(vaddr + kk * 2048, PF_CHUNK, 1024), idesc_o,
                                 (npv | kk) != 0);
                  umma_commit(&bars->o_full[ob]);
                  umma_commit(&bars->kv_empty[vs]);
                  ++cnt.o;
                  ++npv;
                  moved = true;
                }
              }
              if (moved) {
                t_last = clock64();
              } else if (*abortp || clock64() - t_last > LB_SPIN_LIMIT_CYCLES) {
                if (!*abortp) report(p.status, LB_DEV_TIMEOUT);
                ok = false;
                break;
              }
            }
            cnt.kv = base + ntiles;
            cnt.kv2 = vbase + ntiles;
            if (!ok) { *abortp = 1; break; }
            continue;
          }
          for (int j = 0; j <= ntiles && ok; ++j) {
            if (j < ntiles) {
              // ---- S_j  (prefill: K ring; decode: unified ring)
              const uint32_t kp = prefill ? base + j : base + dec_pos_k(j);
              const int ring = prefill ? PF_KSLOTS : nslots;
              const int ks = kp % ring;
              const int sb = cnt.s & 1;
              if (!mbar_wait(&bars->s_empty[sb], ((cnt.s >> 1) & 1) ^ 1, p.status) ||
                  !mbar_wait(&bars->kv_full[ks], (kp / ring) & 1, p.status)) { ok = false; break; }
              tc_fence_after();
              const uint32_t kaddr = prefill ? smem_u32(smem + PF_K_OFF + ks * PF_TILE)
                                             : smem_u32(kv_base + ks * POD_TILE);
              if (prefill) {
                const uint32_t d = tmem + sb * PF_KV;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                  for (int kk = 0; kk < 4; ++kk)
                    umma_bf16(d, umma_desc_sw128(qaddr + c * POD_CHUNK + kk * 32, 16, 1024),
                              umma_desc_sw128(kaddr + c * PF_CHUNK + kk * 32, 16, 1024), idesc_s,
                              (c | kk) != 0);
              } else {
                // four independent accumulators (one per 64-dim chunk) keep the chain of
                // dependent N=16 MMAs short; the softmax threads add them up
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                  for (int c = 0; c < 4; ++c)
                    umma_bf16(tmem + DEC_S_COL + sb * 64 + c * 16,
                              umma_desc_sw128(kaddr + c * POD_CHUNK + kk * 32, 16, 1024),
                              umma_desc_sw128(qaddr + c * 2048 + kk * 32, 16, 1024), idesc_s,
                              kk != 0);
              }
              umma_commit(&bars->s_full[sb]);
              umma_commit(&bars->kv_empty[ks]);
              if (prefill && j == ntiles - 1) umma_commit(&bars->q_empty);
              ++cnt.s;
            }
            if (j > 0) {
              // ---- PV_{j-1}  (prefill: V ring; decode: unified ring)
              const int jj = j - 1;
              const uint32_t vp = prefill ? vbase + jj : base + dec_pos_v(jj, ntiles);
              const int ring = prefill ? PF_VSLOTS : nslots;
              const int vs = (prefill ? PF_KSLOTS : 0) + (int)(vp % ring);
              const int ob = cnt.o & 1;
              if (!mbar_wait(&bars->p_full[ob], (cnt.o >> 1) & 1, p.status) ||
                  !mbar_wait(&bars->kv_full[vs], (vp / ring) & 1, p.status)) { ok = false; break; }
              tc_fence_after();
              const uint32_t vaddr = prefill ? smem_u32(smem + PF_V_OFF + (vp % ring) * PF_TILE)
                                             : smem_u32(kv_base + vs * POD_TILE);
              if (prefill) {
                // A = P from TMEM: 16 keys (8 columns) per MMA
                const uint32_t pcol = tmem + PF_P_COL + ob * (PF_KV / 2);
                const uint32_t d = tmem + 256;
#pragma unroll
                for (int kk = 0; kk < PF_KV / 16; ++kk)
                  umma_bf16_ts(d, pcol + kk * 8,
                               umma_desc_sw128(vaddr + kk * 2048, PF_CHUNK, 1024), idesc_o,
                               (jj | kk) != 0);
              } else {
                const uint32_t paddr =
                    smem_u32(smem + DEC_SLOTS * POD_TILE + 2 * POD_QD_BYTES + ob * POD_PD_BYTES);
                // per half of the dims, four token-quarter accumulators (independent chains
                // of two MMAs); the softmax threads add them up with the running O
#pragma unroll
                for (int k2 = 0; k2 < 2; ++k2)
#pragma unroll
                  for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      const int kk = 2 * q + k2;
                      umma_bf16(tmem + DEC_O_COL + ob * 128 + h * 64 + q * 16,
                                umma_desc_sw128(vaddr + h * 2 * POD_CHUNK + kk * 2048, POD_CHUNK, 1024),
                                umma_desc_sw128(paddr + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024),
                                idesc_o, k2 != 0);
                    }
              }
              umma_commit(&bars->o_full[ob]);
              umma_commit(&bars->kv_empty[vs]);
              ++cnt.o;
            }
          }
          if (prefill) {
            cnt.kv = base + ntiles;
            cnt.kv2 = vbase + ntiles;
          } else {
            cnt.kv = base + 2 * ntiles;
          }
          if (!ok) { *abortp = 1; break; }
        }
        // every commit issued above has arrived once this one has: the barriers can be
        // re-initialised for the next pass without a late arrive landing on them
        umma_commit(&bars->drain);
        mbar_wait(&bars->drain, 0, p.status);
      }
    } else {
      // ============================================================ softmax / epilogue
      const int wg = (warp - 2) >> 2;        // warpgroup 0 or 1
      const int quad = warp & 3;
      const int row = quad * 32 + lane;
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
      const int tid = threadIdx.x - 64 - 128 * wg;
      const int nthr = prefill ? 256 : 128;   // threads taking part in this mode
      // The softmax threads of a mode meet at every named barrier, also after a failed
      // wait: waits are warp-uniform (mbar_wait_warp) and every exit from the item loop
      // is decided at a barrier that ORs the failures, so no thread is left waiting at a
      // barrier the others have passed.
      while (prefill || wg == 0) {
        const int islot = cnt.item & 1;
        const uint32_t iph = (cnt.item >> 1) & 1;
        const bool got = mbar_wait_warp(&bars->item_full[islot], iph, p.status);
        const int4 it = got ? bars->items[islot] : make_int4(-1, 0, 0, 0);
        ++cnt.item;
        if (!got) *abortp = 1;
        if (named_bar_any(4, nthr, !got || it.x < 0 || *abortp)) break;
        const int b = it.x;
        const int ctx = p.context_lens[b];
        const int q0 = p.cu_seqlens_q[b];
        const int qlen = p.cu_seqlens_q[b + 1] - q0;
        bool ok = true;
        if (prefill) {
          // ---------------------------------------------------- prefill item
          const int h = it.y, qt = it.z;
          const int qrow = qt * POD_KV + row;
          const bool rvalid = qrow < qlen;
          const int pos = rvalid ? ctx - qlen + qrow : -1;   // last visible key
          const int kv_end = min(ctx, ctx - qlen + (qt + 1) * POD_KV);
          const int ntiles = (kv_end + PF_KV - 1) / PF_KV;
          float m = -INFINITY, l = 0.f;
          const uint32_t vbase = cnt.kv2;
          cnt.kv += ntiles;
          cnt.kv2 += ntiles;
          const uint32_t pv0 = cnt.o;  // global index of this item's first PV
          cnt.o += ntiles;
          for (int j = 0; j < ntiles; ++j) {
            const uint32_t pv = pv0 + j;
            const int sb = cnt.s & 1;
            if (!mbar_wait_warp(&bars->s_full[sb], (cnt.s >> 1) & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            // both warpgroups read the whole score row (for the row max); each then
            // exponentiates and writes its own half of the keys
            constexpr int HALF = PF_KV / 2;
            float s[HALF], so[HALF];
            {
              uint32_t r[32], ro[32];
              tmem_ld32(tl + sb * PF_KV + wg * HALF, r);
              tmem_ld32(tl + sb * PF_KV + (wg ^ 1) * HALF, ro);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                s[i] = __uint_as_float(r[i]);
                so[i] = __uint_as_float(ro[i]);
              }
            }
            tc_fence_before();
            mbar_arrive(&bars->s_empty[sb]);
            ++cnt.s;
            const int k0 = j * PF_KV + wg * HALF;
            const int ko = j * PF_KV + (wg ^ 1) * HALF;
            float mx[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mx[u] = -INFINITY;
            if (j * PF_KV + PF_KV - 1 <= pos) {   // whole tile visible: no masking
#pragma unroll
              for (int i = 0; i < HALF; ++i) {
                mx[i & 7] = fmaxf(mx[i & 7], s[i]);
                mx[(i + 4) & 7] = fmaxf(mx[(i + 4) & 7], so[i]);
              }
            } else {
#pragma unroll
              for (int i = 0; i < HALF; ++i) {
                s[i] = (k0 + i <= pos) ? s[i] : -INFINITY;
                mx[i & 7] = fmaxf(mx[i & 7], s[i]);
                mx[(i + 4) & 7] = fmaxf(mx[(i + 4) & 7], (ko + i <= pos) ? so[i] : -INFINITY);
              }
            }
            float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            mt = (mt == -INFINITY) ? -INFINITY : mt * p.scale_log2;   // scale > 0 keeps order
            // Lazy rescaling: the exponent base m moves only when the row max exceeds it by
            // more than 8 (log2 units), so p = 2^(s - m) <= 256 stays exact in fp32/bf16
            // and O in TMEM is rescaled rarely.  The final O / l uses the same m, so the
            // result is unchanged.
            float alpha = 1.f;
            if (mt > m + 8.f) {
              alpha = (m == -INFINITY) ? 1.f : exp2_approx(m - mt);
              m = mt;
            }
            const float msub = (m == -INFINITY) ? 0.f : m;
            float sm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) sm[u] = 0.f;
#pragma unroll
            for (int i = 0; i < HALF; ++i) {
              s[i] = exp2_approx(fmaf(s[i], p.scale_log2, -msub));   // 2^(-inf) = 0 if masked
              sm[i & 7] += s[i];
            }
            l = l * alpha + (((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7])));
            // P buffer (pv & 1) was last read by PV pv-2; O may be rescaled only once PV pv-1
            // has finished accumulating into it
            const bool rescale = (j > 0) && __any_sync(0xffffffffu, alpha != 1.f);
            if (j >= 2 || (rescale && j >= 1)) {
              const uint32_t need = rescale ? pv - 1 : pv - 2;
              if (!mbar_wait_warp(&bars->o_full[need & 1], (need >> 1) & 1, p.status)) { ok = false; break; }
              tc_fence_after();
            }
            {
              // this warpgroup's 32 keys of the row, two per column, into P buffer (pv & 1)
              uint32_t pk[HALF / 2];
#pragma unroll
              for (int c = 0; c < HALF / 2; ++c) pk[c] = pack_bf16x2(s[2 * c], s[2 * c + 1]);
              tmem_st16(tl + PF_P_COL + (pv & 1) * (PF_KV / 2) + wg * (HALF / 2), pk);
            }
            if (rescale) {   // this warpgroup's half of the O columns
#pragma unroll 1
              for (int c = 0; c < 4; ++c) {
                uint32_t r[32];
                tmem_ld32(tl + 256 + wg * 128 + c * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                tmem_st32(tl + 256 + wg * 128 + c * 32, r);
              }
              tmem_wait_st();
            }
            // keys past the context in the last tile may hold stale (even NaN) cache
            // bytes; P is 0 there, but 0 * NaN would poison O, so zero those V rows
            if (j * PF_KV + PF_KV > ctx) {
              const uint32_t vp = vbase + j;
              if (!mbar_wait_warp(&bars->kv_full[PF_KSLOTS + vp % PF_VSLOTS], (vp / PF_VSLOTS) & 1, p.status)) { ok = false; break; }
              if (wg == 0 && row < PF_KV && j * PF_KV + row >= ctx) {
                const uint32_t v = smem_u32(smem + PF_V_OFF + (vp % PF_VSLOTS) * PF_TILE) + row * 128;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                  for (int u = 0; u < 8; ++u) st_shared_v4(v + c * PF_CHUNK + u * 16, 0, 0, 0, 0);
              }
            }
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&bars->p_full[pv & 1]);
          }
          // last PV (completion implies all earlier ones)
          if (ok) {
            const uint32_t last = cnt.o - 1;
            ok = mbar_wait_warp(&bars->o_full[last & 1], (last >> 1) & 1, p.status);
            tc_fence_after();
          }
          bars->psum[wg][row] = l;
          if (named_bar_any(2, 256, !ok)) { *abortp = 1; break; }
          l += bars->psum[wg ^ 1][row];
          const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
          const long long tok = (long long)q0 + qrow;
          const __nv_bfloat16* grow = p.gate + tok * p.gate_st + (long long)h * p.gate_sh;
          __nv_bfloat16* orow = p.ogated ? p.ogated + tok * (long long)(p.Hq * POD_D) + h * POD_D : nullptr;
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            const int c = wg * 4 + cc;   // this warpgroup's 32-column chunks of O
            uint32_t r[32];
            tmem_ld32(tl + 256 + c * 32, r);
            tmem_wait_ld();
            if (rvalid) {
              float o[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(r[i]) * inv_l;
              if (p.attn_out) {
                uint4* dst = reinterpret_cast<uint4*>(p.attn_out + tok * (long long)(p.Hq * POD_D) +
                                                      h * POD_D + c * 32);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  dst[q] = make_uint4(pack_bf16x2(o[8 * q], o[8 * q + 1]),
                                      pack_bf16x2(o[8 * q + 2], o[8 * q + 3]),
                                      pack_bf16x2(o[8 * q + 4], o[8 * q + 5]),
                                      pack_bf16x2(o[8 * q + 6], o[8 * q + 7]));
              }
              if (p.ogated) {
                // o_proj input: o * sigmoid(gate), or o itself when there is no gate
                float gs[32];
                if (p.gate) {
                  const uint4* gsrc = reinterpret_cast<const uint4*>(grow + c * 32);
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const uint4 g = gsrc[q];
                    gs[8 * q] = sigmoid_f(bf16_lo(g.x));
                    gs[8 * q + 1] = sigmoid_f(bf16_hi(g.x));
                    gs[8 * q + 2] = sigmoid_f(bf16_lo(g.y));
                    gs[8 * q + 3] = sigmoid_f(bf16_hi(g.y));
                    gs[8 * q + 4] = sigmoid_f(bf16_lo(g.z));
                    gs[8 * q + 5] = sigmoid_f(bf16_hi(g.z));
                    gs[8 * q + 6] = sigmoid_f(bf16_lo(g.w));
                    gs[8 * q + 7] = sigmoid_f(bf16_hi(g.w));
                  }
                } else {
#pragma unroll
                  for (int i = 0; i < 32; ++i) gs[i] = 1.f;
                }
                uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  dst[q] = make_uint4(pack_bf16x2(o[8 * q] * gs[8 * q], o[8 * q + 1] * gs[8 * q + 1]),
                                      pack_bf16x2(o[8 * q + 2] * gs[8 * q + 2], o[8 * q + 3] * gs[8 * q + 3]),
                                      pack_bf16x2(o[8 * q + 4] * gs[8 * q + 4], o[8 * q + 5] * gs[8 * q + 5]),
                                      pack_bf16x2(o[8 * q + 6] * gs[8 * q + 6], o[8 * q + 7] * gs[8 * q + 7]));
              }
            }
          }
          tc_fence_before();
        } else {
          // ---------------------------------------------------- decode item
          const bool fine = p.gqa <= 8
              ? dec_softmax_item<8>(p, bars, cnt, smem, kv_base, nslots, tl, quad, lane, row, tid, b, ctx, it.y, it.z, ok)
              : dec_softmax_item<16>(p, bars, cnt, smem, kv_base, nslots, tl, quad, lane, row, tid, b, ctx, it.y, it.z, ok);
          if (!fine) { *abortp = 1; break; }
        }
        // item done: release its descriptor / Q slot (all softmax threads are past it)
        named_bar_sync(3, nthr);
        if (wg == 0 && tid == 0) mbar_arrive(&bars->item_empty[islot]);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int i = 0; i < 5; ++i) {
        mbar_inval(&bars->kv_full[i]);
        mbar_inval(&bars->kv_empty[i]);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_inval(&bars->item_full[i]);
        mbar_inval(&bars->item_empty[i]);
        mbar_inval(&bars->s_full[i]);
        mbar_inval(&bars->s_empty[i]);
        mbar_inval(&bars->p_full[i]);
        mbar_inval(&bars->o_full[i]);
      }
      mbar_inval(&bars->q_empty);
      mbar_inval(&bars->drain);
      // the other queue already handed out every item (or never had any): no second pass
      bars->skip_pass = pf_first ? *(volatile const int*)p.dec_next >= *p.dec_count
                                 : *(volatile const int*)p.pf_next >= *p.pf_count;
    }
    __syncthreads();
    if (*abortp || (pass == 0 && bars->skip_pass)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(bars->tmem_base, POD_TMEM_COLS);
  }
}

}  // namespace lb
