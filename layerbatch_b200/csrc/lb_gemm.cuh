// Persistent GEMM on sm_100a tensor cores: C = A . B^T, bf16 in, f32 accumulate in TMEM,
// with the epilogues of the dense projections (router logits, o_proj and its split-K and
// tensor-parallel forms).  The grouped expert GEMMs live in lb_gemm_tok.cuh.
//
// Layout: A [M, K] and B [N, K] (K contiguous), i.e. activations times an nn.Linear weight.
// Tiles are 128 x BN x 64 (M x N x K); one CTA per SM walks a static tile sequence:
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..5  : epilogue (TMEM -> registers -> global), 1 thread per accumulator row
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps the
// mainloop of tile i+1.  Stages of A/B tiles are 128B-swizzled, K-major.
#pragma once

#include <cuda.h>
#include "lb_common.cuh"
#include "lb_peer.h"
#include "lb_prologue.cuh"

namespace lb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

enum EpiKind : int {
  EPI_BF16 = 0,        // C = bf16(acc)
  EPI_F32_RED = 4,     // out32 += acc (split-K partials, vector reductions)
  EPI_F32_PEER = 5,    // fp32 tile -> inbox of the rank owning its m-tile (tensor parallel);
                       // the last CTA publishes the call's epoch to every rank
  EPI_F32_SPLIT = 6,   // split-K partial ks -> its own fp32 slice out32[ks] (plain stores;
                       // k_splitk_reduce sums the slices in split order: deterministic)
  EPI_QKV = 7,         // q/k/v projection with the attention prologue (qkv_prologue_tile;
                       // BN = 256 = one head row per tile)
};

struct GemmArgs {
  int* status;
  int m;                   // rows of A and C
  int n_tiles;             // N / BN
  int k_blocks;            // K / 64 handled by one split
  int splits;              // split-K factor
  void* out;
  long long ldo;
  int out_rows;            // rows of `out` (bounds check)
  int out_cols;            // columns of `out` (bounds check)
  TpPeers tp;              // EPI_F32_PEER
  LbPrologueArgs pro;      // EPI_QKV
};

constexpr int EPI_STAGE_LD = 36;  // floats per row of the peer-store transpose buffer
constexpr int EPI_STAGE_BYTES = 4 * 32 * EPI_STAGE_LD * 4 + 16;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int TMEM_COLS = 2 * BN;
  static size_t bytes() { return 1024 + (size_t)STAGES * STAGE_BYTES + BAR_BYTES; }
};

struct TileCoord {
  int m, n, ks;
};

// Tile t -> (m-tile, n-tile, split), m fastest, then the split: CTAs that run at the
// same time share the B tile.
__device__ __forceinline__ TileCoord decode_tile(int t, const GemmArgs& p) {
  const int mt = (p.m + GEMM_BM - 1) / GEMM_BM;
  const int rest = t / mt;
  return TileCoord{t % mt, rest / p.splits, rest % p.splits};
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const GemmArgs p) {
  pdl_entry();
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * S::B_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // EPI_F32_PEER: per epilogue warp a 32 x EPI_STAGE_LD fp32 transpose buffer
  float* s_stage = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + S::BAR_BYTES);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total =
      p.m > 0 ? ((p.m + GEMM_BM - 1) / GEMM_BM) * p.n_tiles * p.splits : 0;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < total && !*s_abort; t += gridDim.x) {
        const TileCoord c = decode_tile(t, p);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status)) { *s_abort = 1; break; }
          mbar_arrive_expect_tx(&full[stage], S::STAGE_BYTES);
          const int kc = (c.ks * p.k_blocks + kb) * GEMM_BK;
          tma_load_2d(sA + stage * S::A_BYTES, &tmA, &full[stage], kc, c.m * GEMM_BM);
          tma_load_3d(sB + stage * S::B_BYTES, &tmB, &full[stage], kc, c.n * BN, 0);
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
    constexpr uint32_t IDESC = umma_idesc_bf16(GEMM_BM, BN, false, false);
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total && !*s_abort; t += gridDim.x) {
        if (!mbar_wait(&tempty[buf], aphase ^ 1, p.status)) { *s_abort = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) { *s_abort = 1; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * S::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * S::B_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (*s_abort) break;
        umma_commit(&tfull[buf]);
        buf ^= 1;
        if (buf == 0) aphase ^= 1;
      }
      if (*s_abort && issued_any) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    int buf = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < total && !*s_abort; t += gridDim.x) {
      const TileCoord c = decode_tile(t, p);
      if (!mbar_wait(&tfull[buf], aphase, p.status)) { *s_abort = 1; break; }
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * BN;

      const int valid_rows = p.m - c.m * GEMM_BM;
      const int out_row = c.m * GEMM_BM + row_in_tile;
      const bool row_ok = row_in_tile < valid_rows && out_row < p.out_rows;

      if constexpr (EPI == EPI_QKV) {
        static_assert(EPI != EPI_QKV || BN == PRO_D, "EPI_QKV: one 256-dim head row per tile");
        qkv_prologue_tile(p.pro, c.n, tbase, row_ok, out_row, p.out, p.ldo, p.status);
      }
#pragma unroll 1
      for (int ch = 0; ch < (EPI == EPI_QKV ? 0 : BN / 32); ++ch) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tbase + ch * 32, v);
        tmem_wait_ld();
        const int col = c.n * BN + ch * 32;
        if constexpr (EPI == EPI_F32_PEER) {
          // Rank s's partial of a row goes to region s of the inbox of the rank owning
          // the row's m-tile.  The warp's 32 x 32 fp32 block is transposed through
          // shared memory so that every store writes 128-byte row segments (8 lanes per
          // row): large NVLink writes instead of 16-byte ones.
          float* stg = s_stage + quad * (32 * EPI_STAGE_LD);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(stg + lane * EPI_STAGE_LD + 4 * i) =
                make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                            __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          __syncwarp();
          const int owner = c.m % p.tp.size;
          float* inbox = p.tp.inbox[0];
#pragma unroll
          for (int r = 1; r < LB_PEER_MAX; ++r)
            if (r == owner) inbox = p.tp.inbox[r];
          const int warp_row0 = quad * 32;            // first tile row of this warp
          const long long row0 = (long long)(out_row - row_in_tile) + warp_row0;
          const int cc = (lane & 7) * 4;
#pragma unroll
          for (int jr = 0; jr < 8; ++jr) {
            const int r = 4 * jr + (lane >> 3);
            const float4 val = *reinterpret_cast<const float4*>(stg + r * EPI_STAGE_LD + cc);
            if (warp_row0 + r < valid_rows && row0 + r < p.out_rows && col + 32 <= p.out_cols)
              *reinterpret_cast<float4*>(
                  inbox + ((long long)p.tp.rank * p.tp.inbox_rows + row0 + r) * p.ldo + col + cc) = val;
          }
          __syncwarp();
          continue;
        }
        if (!row_ok || col + 32 > p.out_cols) {
          // nothing to store for this row / chunk
        } else if constexpr (EPI == EPI_F32_SPLIT) {
          float* out = reinterpret_cast<float*>(p.out) +
                       ((long long)c.ks * p.out_rows + out_row) * p.ldo + col;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(out + 4 * i) =
                make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                            __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        } else if constexpr (EPI == EPI_F32_RED) {
          float* out = reinterpret_cast<float*>(p.out) + (long long)out_row * p.ldo + col;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            red_add_v4_f32(out + 4 * i, __uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                           __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        } else {
          float f[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
          uint4* dst = reinterpret_cast<uint4*>(out + (long long)out_row * p.ldo + col);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pack_bf16x2(f[8 * i], f[8 * i + 1]),
                                pack_bf16x2(f[8 * i + 2], f[8 * i + 3]),
                                pack_bf16x2(f[8 * i + 4], f[8 * i + 5]),
                                pack_bf16x2(f[8 * i + 6], f[8 * i + 7]));
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      buf ^= 1;
      if (buf == 0) aphase ^= 1;
    }
  }

  if constexpr (EPI == EPI_F32_PEER) {
    // every tile of this CTA is stored: the last CTA to get here tells every rank that
    // this rank's partials of the call are in place
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* own = p.tp.hdr[p.tp.rank];
      if (atomicAdd(own + TPH_DONE_GEMM, 1) == (int)gridDim.x - 1) {
        __threadfence_system();
        const int epoch = own[TPH_EPOCH] + 1;
        own[TPH_EPOCH] = epoch;
        own[TPH_DONE_GEMM] = 0;
        for (int r = 0; r < p.tp.size; ++r) st_release_sys(p.tp.hdr[r] + TPH_PART + p.tp.rank, epoch);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}


// ------------------------------------------------------------------------------ CTA pair
// The same C = A . B^T on a cluster of two CTAs (cta_group::2): the pair computes a
// 256 x 256 tile with one M = 256 MMA per K step.  Each CTA loads its own 128 rows of A and
// 128 of the 256 B rows (32 KB per k-block instead of the 48 KB a 128 x 256 tile needs
// alone, so each SM reads a third less from L2 per FLOP and six stages fit), and its TMEM
// receives its 128 accumulator rows, which its own epilogue stores.
//   warp 0 (both CTAs) : TMA producer; the loads of both CTAs complete on the first CTA's
//                        `full` barrier, which expects the pair's bytes
//   warp 1             : pair TMEM allocation (both CTAs); MMA issue (first CTA only), with
//                        each commit sent to the barrier of both CTAs
//   warps 2..          : epilogue of this CTA's rows, EPW warps: with 4 one warp per TMEM
//                        lane quadrant drains both accumulators in turn; with 8 (the q/k/v
//                        prologue epilogue, longer than a tile's mainloop) warps 2-5 drain
//                        accumulator 0 and warps 6-9 accumulator 1, so each group has two
//                        mainloops' time per tile; one arrival per warp on the first CTA's
//                        `tempty` barrier (eight per tile)
// Every wait is bounded; the CTAs meet in cluster barriers after the barrier set-up and
// before the TMEM release, so neither leaves while the other may still signal it.
constexpr int PAIR_BN = 256;

template <int STAGES>
struct PairSmem {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;          // this CTA's 128 A rows
  static constexpr int B_BYTES = (PAIR_BN / 2) * GEMM_BK * 2;    // this CTA's 128 B rows
  static constexpr int BAR_BYTES = 256;
  static constexpr int TMEM_COLS = 2 * PAIR_BN;                  // two accumulators
  static size_t bytes() { return 1024 + (size_t)STAGES * (A_BYTES + B_BYTES) + BAR_BYTES; }
};

template <int STAGES, int EPI, int EPW>
__global__ void __launch_bounds__(64 + 32 * EPW, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmArgs p) {
  static_assert(EPI == EPI_BF16 || EPI == EPI_QKV, "pair GEMM epilogues: bf16 and q/k/v");
  static_assert(EPI != EPI_QKV || PAIR_BN == PRO_D, "EPI_QKV: one 256-dim head row per tile");
  static_assert(EPW == 4 || EPW == 8, "one or two epilogue warps per TMEM lane quadrant");
  using S = PairSmem<STAGES>;
  constexpr uint32_t PAIR_TX = 2u * (S::A_BYTES + S::B_BYTES);
  pdl_entry();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * S::B_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();   // 0: issues the MMAs, 1: its peer
  const int cid = blockIdx.x >> 1;           // cluster (2 consecutive CTAs of the 1-D grid)
  const int ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  __syncthreads();
  cluster_sync();   // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int mt2 = (p.m + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
  const int total = p.m > 0 ? mt2 * p.n_tiles : 0;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one_sync()) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = cid; t < total && !*s_abort; t += ncl) {
        const int arow = (t % mt2) * 2 * GEMM_BM + (int)rank * GEMM_BM;
        const int brow = (t / mt2) * PAIR_BN + (int)rank * (PAIR_BN / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status)) { *s_abort = 1; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], PAIR_TX);
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          const int kc = kb * GEMM_BK;
          tma_load_2d_pair(sA + stage * S::A_BYTES, &tmA, fb, kc, arow);
          tma_load_2d_pair(sB + stage * S::B_BYTES, &tmB, fb, kc, brow);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Tail: every stage this CTA filled has been released by the pair's MMAs, i.e. their
      // commits' arrivals on this CTA's `empty` barriers have landed (stages never filled
      // pass at once).  After an abort the waits still end at their time limit.
      for (int i = 0; i < STAGES; ++i) {
        mbar_wait(&empty[stage], phase ^ 1, nullptr);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = umma_idesc_bf16(2 * GEMM_BM, PAIR_BN, false, false);
    if (rank == 0 && elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int t = cid; t < total && !*s_abort; t += ncl) {
        if (!mbar_wait(&tempty[buf], aphase ^ 1, p.status)) { *s_abort = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * PAIR_BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) { *s_abort = 1; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * S::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * S::B_BYTES);
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k) {
            const uint64_t ad = umma_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(b0 + k * 32, 16, 1024);
            umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          const uint32_t e = smem_u32(&empty[stage]);
          umma_commit_pair(mapa_shared(e, 0));
          umma_commit_pair(mapa_shared(e, 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (*s_abort) break;
        const uint32_t f = smem_u32(&tfull[buf]);
        umma_commit_pair(mapa_shared(f, 0));
        umma_commit_pair(mapa_shared(f, 1));
        buf ^= 1;
        if (buf == 0) aphase ^= 1;
      }
      if (*s_abort && issued_any) {
        umma_commit_pair(mapa_shared(smem_u32(drain), 0));
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    constexpr int NG = EPW / 4;            // epilogue groups; group g takes local tiles g, g+NG..
    const int grp = (warp - 2) / 4;
    for (int i = grp;; i += NG) {
      const int t = cid + i * ncl;
      if (t >= total || *s_abort) break;
      const int buf = i & 1;                        // accumulator of the pair's i-th tile
      const uint32_t aphase = (uint32_t)(i >> 1) & 1u;
      if (!mbar_wait(&tfull[buf], aphase, p.status)) { *s_abort = 1; break; }
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * PAIR_BN;
      const int n = t / mt2;
      const int row0 = (t % mt2) * 2 * GEMM_BM + (int)rank * GEMM_BM;
      const int out_row = row0 + row_in_tile;
      const bool row_ok = out_row < p.m && out_row < p.out_rows;
      if constexpr (EPI == EPI_QKV) {
        qkv_prologue_tile(p.pro, n, tbase, row_ok, out_row, p.out, p.ldo, p.status);
      } else {
#pragma unroll 1
        for (int ch = 0; ch < PAIR_BN / 32; ++ch) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tbase + ch * 32, v);
          tmem_wait_ld();
          const int col = n * PAIR_BN + ch * 32;
          if (row_ok && col + 32 <= p.out_cols) {
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
            uint4* dst = reinterpret_cast<uint4*>(out + (long long)out_row * p.ldo + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(
                  pack_bf16x2(__uint_as_float(v[8 * i]), __uint_as_float(v[8 * i + 1])),
                  pack_bf16x2(__uint_as_float(v[8 * i + 2]), __uint_as_float(v[8 * i + 3])),
                  pack_bf16x2(__uint_as_float(v[8 * i + 4]), __uint_as_float(v[8 * i + 5])),
                  pack_bf16x2(__uint_as_float(v[8 * i + 6]), __uint_as_float(v[8 * i + 7])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
    }
  }

  __syncthreads();
  cluster_sync();   // no CTA releases TMEM or exits while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace lb
