// Grouped expert GEMM with the token rows as the MMA N operand (sm_100a tensor cores).
//
// For group g (an expert; group 0 may be the shared expert) with R_g packed token rows:
//     D_g^T[f, t] = sum_k W_g[f, k] * X[row_start[g] + t, k]
// The weights W_g [F, K] (nn.Linear layout, K contiguous) are the 128-row A operand and the
// group's tokens the B operand, so a tile holds up to TN tokens of one expert and the MMA
// width is the group's remaining token count rounded up to 16, not a 128-row M tile:
// an expert with 20 routed rows costs a 32-wide MMA instead of a 128-row one.
//
// A work unit is (group, feature block, token tile).  It drives two accumulators that
// share the token operand:
//   * gate/up (TOK_EPI_SWIGLU): accumulator 0 = gate rows fb*128.., accumulator 1 = the
//     matching up rows, so thread f of the epilogue holds gate and up of feature f and
//     writes act[t, f] = silu(gate) * up;
//   * down (TOK_EPI_SCALE): accumulators 0 / 1 = output features fb*256 + [0,128) /
//     [128,256), written as yw[t, f] = acc * row_scale[t].
// Per k-block the unit loads 256 weight rows and up to TN token rows (in 32-row boxes,
// only as many boxes as the tile has tokens).  Units are ordered feature block fastest,
// so the CTAs that run at the same time share token tiles and expert weights in L2.
//
// One CTA per SM walks a static unit sequence:
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..   : EPW epilogue warps; TMEM lane quadrant (warp & 3) = 32 features per
//                 warp; with 8 warps the two of a quadrant take alternate 32-token chunks
// TMEM holds NBUF x 2 accumulators of TN columns (each starting on a power-of-two
// column); with NBUF = 2 the epilogue of a unit
// overlaps the mainloop of the next.  Every wait is bounded and reports a status code.
#pragma once

#include <cuda.h>
#include "lb_common.cuh"

namespace lb {

constexpr int TOK_MAX_THREADS = 320;  // 2 + 8 warps
constexpr int TOK_FB = 128;   // weight rows (features) per accumulator = MMA M
constexpr int TOK_BOX = 32;   // token rows per TMA box

enum TokEpi : int {
  TOK_EPI_SWIGLU = 0,  // act[t, fb*128 + f] = bf16(silu(acc0[f, t]) * acc1[f, t])
  TOK_EPI_SCALE = 1,   // out[t, col_a(f)] = bf16(acc_a[f, t] * row_scale[t]), a = 0, 1
};

struct TokArgs {
  int* status;
  const int* row_start;  // [G+1] first packed row of every group (row_start[0] = 0)
  int num_groups;        // G
  int n_fb;              // feature blocks per group
  int fb_stride;         // weight rows (and output columns) between feature blocks
  int acc1_off;          // weight row / output column offset of accumulator 1 (routed)
  int acc1_off_sh;       // the same for the shared group (its own weight maps)
  int k_blocks;          // K / 64
  int shared_group;      // group whose weights / tokens come from the *_sh maps (-1: none)
  int w_group_base;      // routed weight depth coordinate = g - w_group_base
  void* out;             // bf16 [out_rows, ldo]; packed row r of group g -> out row r
  long long ldo;
  int out_rows;
  int out_cols;
  const float* row_scale;  // TOK_EPI_SCALE: per packed row
};

template <int TN, int NBUF, int STAGES>
struct TokSmem {
  static constexpr int W_BYTES = 2 * TOK_FB * 64 * 2;  // two 128 x 64 weight tiles
  static constexpr int X_BYTES = TN * 64 * 2;          // TN x 64 token tile
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  // down epilogue: per epilogue warp a 32-token x 32-feature bf16 block (token rows)
  static constexpr int STG_WARP_BYTES = 32 * 32 * 2;
  static constexpr int STG_BYTES = 8 * STG_WARP_BYTES;
  static constexpr int BAR_BYTES = 256;
  // TMEM columns per accumulator: TN rounded up to a power of two, so that every
  // accumulator starts on a power-of-two column
  static constexpr int ACC_COLS = TN <= 32 ? 32 : TN <= 64 ? 64 : TN <= 128 ? 128 : 256;
  static constexpr int TMEM_COLS = 2 * ACC_COLS * NBUF;
  static size_t bytes(int num_groups) {
    return 1024 + (size_t)STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES +
           4 * (2 * (size_t)num_groups + 4) + 4 * TOK_MAX_THREADS;
  }
};

struct TokUnit {
  int g, fb, tt;
};

// Unit u -> (group, feature block, token tile).  s_ut[g] is the first unit of group g.
__device__ __forceinline__ TokUnit tok_unit(int u, const int* s_ut, int G, int n_fb) {
  int lo = 0, hi = G - 1;  // largest g with s_ut[g] <= u (skips groups without units)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_ut[mid] <= u) lo = mid; else hi = mid - 1;
  }
  const int l = u - s_ut[lo];
  return TokUnit{lo, l % n_fb, l / n_fb};
}

template <int TN, int NBUF, int STAGES, int EPI, int EPW>
__global__ void __launch_bounds__(64 + 32 * EPW, 1)
    k_gemm_tok(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmW_sh0,
               const __grid_constant__ CUtensorMap tmW_sh1, const __grid_constant__ CUtensorMap tmX,
               const __grid_constant__ CUtensorMap tmX_sh, const TokArgs p) {
  static_assert(TN % TOK_BOX == 0 && TN >= 32 && TN <= 256, "token tile");
  using S = TokSmem<TN, NBUF, STAGES>;
  static_assert(S::TMEM_COLS <= 512 && NBUF >= 1, "TMEM columns");
  static_assert(EPW == 4 || EPW == 8, "epilogue warps: one or two per TMEM lane quadrant");
  constexpr int THREADS = 64 + 32 * EPW;
  pdl_entry();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * S::W_BYTES;
  uint8_t* sStg = sX + STAGES * S::X_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + S::STG_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int G = p.num_groups;
  int* s_rs = reinterpret_cast<int*>(bars) + S::BAR_BYTES / 4;  // [G+1] row starts
  int* s_ut = s_rs + G + 1;                                     // [G+1] unit starts
  int* s_part = s_ut + G + 1;                                   // [THREADS] scan

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * EPW);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = tid; i <= G; i += THREADS) s_rs[i] = p.row_start[i];
  __syncthreads();
  // units per group = n_fb * ceil(rows / TN); exclusive scan over the groups
  {
    const int per = (G + THREADS - 1) / THREADS;
    const int g0 = tid * per, g1 = min(G, g0 + per);
    int loc = 0;
    for (int g = g0; g < g1; ++g) loc += (s_rs[g + 1] - s_rs[g] + TN - 1) / TN;
    s_part[tid] = loc;
    __syncthreads();
    if (tid == 0) {
      int run = 0;
      for (int i = 0; i < THREADS; ++i) {
        const int v = s_part[i];
        s_part[i] = run;
        run += v;
      }
      s_ut[G] = run * p.n_fb;
    }
    __syncthreads();
    int run = s_part[tid];
    for (int g = g0; g < g1; ++g) {
      s_ut[g] = run * p.n_fb;
      run += (s_rs[g + 1] - s_rs[g] + TN - 1) / TN;
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = s_ut[G];

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      prefetch_tmap(&tmW);
      prefetch_tmap(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int u = blockIdx.x; u < total && !*s_abort; u += gridDim.x) {
        const TokUnit c = tok_unit(u, s_ut, G, p.n_fb);
        const bool sh = (c.g == p.shared_group);
        const int nv = min(TN, s_rs[c.g + 1] - s_rs[c.g] - c.tt * TN);
        const int nbox = (nv + TOK_BOX - 1) / TOK_BOX;
        const int xrow = s_rs[c.g] + c.tt * TN;
        const int wr0 = c.fb * p.fb_stride;
        const int wr1 = wr0 + (sh ? p.acc1_off_sh : p.acc1_off);
        const int depth = sh ? 0 : c.g - p.w_group_base;
        const void* w0 = sh ? (const void*)&tmW_sh0 : (const void*)&tmW;
        const void* w1 = sh ? (const void*)&tmW_sh1 : (const void*)&tmW;
        const void* xm = sh ? (const void*)&tmX_sh : (const void*)&tmX;
        const uint32_t tx = (uint32_t)S::W_BYTES + (uint32_t)nbox * TOK_BOX * 128u;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status)) { *s_abort = 1; break; }
          mbar_arrive_expect_tx(&full[stage], tx);
          const int kc = kb * 64;
          uint8_t* dW = sW + stage * S::W_BYTES;
          tma_load_3d(dW, w0, &full[stage], kc, wr0, depth);
          tma_load_3d(dW + S::W_BYTES / 2, w1, &full[stage], kc, wr1, depth);
          uint8_t* dX = sX + stage * S::X_BYTES;
          for (int b = 0; b < nbox; ++b)
            tma_load_2d(dX + b * TOK_BOX * 128, xm, &full[stage], kc, xrow + b * TOK_BOX);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*s_abort) {
        // Let copies already in flight land before the CTA can exit (bounded).
        int st = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--st < 0) { st = STAGES - 1; ph ^= 1; }
          mbar_wait(&full[st], ph, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int u = blockIdx.x; u < total && !*s_abort; u += gridDim.x) {
        const TokUnit c = tok_unit(u, s_ut, G, p.n_fb);
        const int nv = min(TN, s_rs[c.g + 1] - s_rs[c.g] - c.tt * TN);
        const uint32_t idesc = umma_idesc_bf16(TOK_FB, (nv + 15) & ~15, false, false);
        if (!mbar_wait(&tempty[buf], aphase ^ 1, p.status)) { *s_abort = 1; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + buf * 2 * S::ACC_COLS;
        const uint32_t d1 = d0 + S::ACC_COLS;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) { *s_abort = 1; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sW + stage * S::W_BYTES);
          const uint32_t a1 = a0 + S::W_BYTES / 2;
          const uint32_t b0 = smem_u32(sX + stage * S::X_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            umma_bf16(d0, umma_desc_sw128(a0 + k * 32, 16, 1024), bd, idesc, acc);
            umma_bf16(d1, umma_desc_sw128(a1 + k * 32, 16, 1024), bd, idesc, acc);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (*s_abort) break;
        umma_commit(&tfull[buf]);
        if (++buf == NBUF) { buf = 0; aphase ^= 1; }
      }
      if (*s_abort && issued_any) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3;            // TMEM lane quadrant this warp may access
    const int f_in = quad * 32 + lane;    // feature of this thread within an accumulator
    const int part = (warp - 2) / 4;      // with 8 warps, two share a quadrant's chunks
    constexpr int NPART = EPW / 4;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    int buf = 0;
    uint32_t aphase = 0;
    for (int u = blockIdx.x; u < total && !*s_abort; u += gridDim.x) {
      const TokUnit c = tok_unit(u, s_ut, G, p.n_fb);
      const bool sh = (c.g == p.shared_group);
      const int nv = min(TN, s_rs[c.g + 1] - s_rs[c.g] - c.tt * TN);
      const long long row0 = (long long)s_rs[c.g] + (long long)c.tt * TN;
      if (!mbar_wait(&tfull[buf], aphase, p.status)) { *s_abort = 1; break; }
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * 2 * S::ACC_COLS;
      const int nch = (nv + 31) / 32;
      if constexpr (EPI == TOK_EPI_SWIGLU) {
        const int col = c.fb * p.fb_stride + f_in;
        const bool col_ok = col < p.out_cols;
#pragma unroll 1
        for (int ch = part; ch < nch; ch += NPART) {
          uint32_t g[32], v[32];
          __syncwarp();
          tmem_ld32(tb + ch * 32, g);
          tmem_ld32(tb + S::ACC_COLS + ch * 32, v);
          tmem_wait_ld();
          const int nj = min(32, nv - ch * 32);
          const long long r0 = row0 + ch * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < nj && col_ok && r0 + j < p.out_rows) {
              const float a = silu_f(__uint_as_float(g[j])) * __uint_as_float(v[j]);
              out[(r0 + j) * p.ldo + col] = __float2bfloat16_rn(a);
            }
          }
        }
      } else {
        // The warp's 32 features x 32 tokens of a chunk become token rows through its own
        // 2 KB shared block: 2-byte shared stores (one token per instruction, 64 contiguous
        // bytes), then per lane 16-byte loads and 16-byte global stores (four lanes per
        // token's 64 bytes), an eighth of the store instructions of per-feature stores.
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(sStg + (warp - 2) * S::STG_WARP_BYTES);
        const int f8 = (lane & 3) * 8;   // this lane's 8 features of a token row
#pragma unroll 1
        for (int a = 0; a < 2; ++a) {
          const int col0 = c.fb * p.fb_stride + (a ? (sh ? p.acc1_off_sh : p.acc1_off) : 0) + quad * 32;
          const bool col_ok = col0 + f8 + 8 <= p.out_cols;
#pragma unroll 1
          for (int ch = part; ch < nch; ch += NPART) {
            uint32_t v[32];
            __syncwarp();   // the previous chunk's shared reads are done
            tmem_ld32(tb + a * S::ACC_COLS + ch * 32, v);
            tmem_wait_ld();
            const int nj = min(32, nv - ch * 32);
            const long long r0 = row0 + ch * 32;
            const float s_mine =
                (lane < nj && r0 + lane < p.out_rows) ? p.row_scale[r0 + lane] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float s = __shfl_sync(0xffffffffu, s_mine, j);
              stg[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]) * s);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int j = 8 * i + (lane >> 2);
              const uint4 val = *reinterpret_cast<const uint4*>(stg + j * 32 + f8);
              if (j < nj && col_ok && r0 + j < p.out_rows)
                *reinterpret_cast<uint4*>(out + (r0 + j) * p.ldo + col0 + f8) = val;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      if (++buf == NBUF) { buf = 0; aphase ^= 1; }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace lb
