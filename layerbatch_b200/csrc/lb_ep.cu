// Expert-parallel MoE block over NVLink peer memory (sm_100a).
//
// P ranks of one node; rank r holds experts [r*E/P, (r+1)*E/P) and one exchange buffer
// that every rank maps (CUDA IPC).  Buffer of rank r:
//   header   ints: disp flag [s], return flag [o], row count [s], epoch, CTA counters
//   recv_x   [P][C][H] bf16   rows source s sent to r (region s, its slots in order)
//   recv_ids [P][C][k] int32  the k global expert ids of each of those rows
//   recv_w   [P][C][k] f32    and their routing weights
//   ret_y    [P][C][H] bf16   region o: owner o's per-row sums for r's tokens
// One call = three stream-ordered phases on every rank:
//   dispatch  router GEMM + top-k, routing table (one slot per token and destination rank
//             owning >= 1 of its experts), every token row written once per such rank
//             straight into the owner's recv region, then counts + epoch flag published
//   experts   wait for all sources' flags; grouped gate/up + down GEMMs over the shared
//             expert (own tokens) and the local experts (received rows); each received
//             row's local pairs summed and written back into the source's ret region,
//             then the epoch flag of the return
//   combine   wait for all owners' return flags; out[t] = shared row + returned rows
// Flags carry a per-call epoch (every rank makes the same calls); a kernel that waits on
// another GPU spins with a bounded time limit and records LB_DEV_TIMEOUT instead of
// hanging.  The data-dependent writes of each phase are ordered before its flag by
// system-scope fences and a last-CTA-publishes pattern.
#include <algorithm>
#include <cstring>

#include "lb_gemm_launch.cuh"
#include "lb_host.h"
#include "lb_moe_core.h"

namespace lb {

// Header ints; each group sits on its own 128-byte line.
constexpr int EPH_DISP = 0;        // [s]: epoch of the last dispatch received from rank s
constexpr int EPH_RET = 32;        // [o]: epoch of the last return received from owner o
constexpr int EPH_COUNT = 64;      // [s]: rows rank s sent in its last dispatch
constexpr int EPH_EPOCH = 96;      // this rank's call counter (own GPU only)
constexpr int EPH_DONE_DISP = 128; // CTA completion counters (own GPU only)
constexpr int EPH_DONE_RET = 160;
constexpr size_t EP_HEADER_BYTES = 4096;

struct EpLayout {
  size_t x, ids, w, ret, total;
};

static EpLayout ep_layout(size_t P, size_t C, size_t H, size_t k) {
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  EpLayout L;
  L.x = EP_HEADER_BYTES;
  L.ids = al(L.x + P * C * H * 2);
  L.w = al(L.ids + P * C * k * 4);
  L.ret = al(L.w + P * C * k * 4);
  L.total = al(L.ret + P * C * H * 2);
  return L;
}

struct EpPeers {
  uint8_t* p[LB_EP_MAX_RANKS];
};

// ------------------------------------------------------------------------------ route
// Destination mask of every token (bit r: rank r owns >= 1 of its k experts), one warp per
// token: lane j maps id j through the placement table, the warp ORs the ranks.
__global__ void __launch_bounds__(256) k_ep_mask(const int32_t* __restrict__ ids, int T, int k,
                                                 int epr, int P, const int32_t* __restrict__ expert_slot,
                                                 uint8_t* __restrict__ mask, int* status) {
  pdl_entry();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  unsigned bit = 0;
  for (int j = lane; j < k; j += 32) {
    int e = ids[(long long)t * k + j];
    if (expert_slot && e >= 0 && e < epr * P) e = expert_slot[e];
    const int r = e >= 0 ? e / epr : -1;
    if (r < 0 || r >= P) {
      report(status, LB_DEV_BAD_INDEX);
      continue;
    }
    bit |= 1u << r;
  }
  const unsigned m = __reduce_or_sync(0xffffffffu, bit);
  if (lane == 0) mask[t] = (uint8_t)m;
}

// One block of 1024 threads over the masks.  slot[t][r] = rank of token t among the tokens
// that send a row to rank r (token order), -1 if none; send_count[r] = rows sent to r.
__global__ void __launch_bounds__(1024) k_ep_route(const uint8_t* __restrict__ mask, int T, int P,
                                                   int32_t* __restrict__ slot,
                                                   int* __restrict__ send_count) {
  pdl_entry();
  __shared__ int s_w[32][LB_EP_MAX_RANKS];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (T + 1023) / 1024;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  int cnt[LB_EP_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < LB_EP_MAX_RANKS; ++r) cnt[r] = 0;
  for (int t = t0; t < t1; ++t) {
    const unsigned m = mask[t];
#pragma unroll
    for (int r = 0; r < LB_EP_MAX_RANKS; ++r) cnt[r] += (m >> r) & 1u;
  }
  int incl[LB_EP_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < LB_EP_MAX_RANKS; ++r) {
    int v = cnt[r];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    incl[r] = v;
    if (lane == 31) s_w[wid][r] = v;
  }
  __syncthreads();
  if (wid == 0) {
#pragma unroll
    for (int r = 0; r < LB_EP_MAX_RANKS; ++r) {
      const int v = s_w[lane][r];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += n;
      }
      s_w[lane][r] = x - v;
      if (lane == 31 && r < P) send_count[r] = x;
    }
  }
  __syncthreads();
  int base[LB_EP_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < LB_EP_MAX_RANKS; ++r) base[r] = s_w[wid][r] + incl[r] - cnt[r];
  for (int t = t0; t < t1; ++t) {
    const unsigned m = mask[t];
    for (int r = 0; r < P; ++r) slot[(long long)t * P + r] = ((m >> r) & 1u) ? base[r]++ : -1;
  }
}

// ------------------------------------------------------------------------------ dispatch
struct EpDispatch {
  const __nv_bfloat16* x;
  const int32_t* ids;
  const float* wf;
  const int32_t* slot;
  const int* send_count;
  int T, H, k, P, C, rank;
  unsigned long long off_x, off_ids, off_w;
  EpPeers peers;
  int* status;
};

// One warp per token: its row is read once (all of a lane's 16-byte pieces in flight
// together) and stored to every destination rank's recv region (NVLink stores for other
// ranks), with the k ids and weights.  Token t visits its destinations starting at rank
// (t + rank) % P, so at any moment the warps of every GPU spread their stores over all
// destinations instead of all GPUs writing into the same one.  The last CTA to finish
// publishes the row counts and this call's epoch to every destination.
template <int MAXS>  // H <= MAXS * 256
__global__ void __launch_bounds__(256) k_ep_dispatch(const EpDispatch d) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x / 32;
  const int nvec = d.H / 8;
  const int stripes = d.H / 256;
  for (int t = blockIdx.x * wpb + (int)(threadIdx.x >> 5); t < d.T; t += gridDim.x * wpb) {
    int sl[LB_EP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < LB_EP_MAX_RANKS; ++r)
      sl[r] = r < d.P ? d.slot[(long long)t * d.P + r] : -1;
    const uint4* src = reinterpret_cast<const uint4*>(d.x + (long long)t * d.H) + lane;
    uint4 v[MAXS];
#pragma unroll
    for (int u = 0; u < MAXS; ++u)
      if (u < stripes) v[u] = src[u * 32];
    // destinations in the order r0, r0 + 1, ..., P - 1, 0, ..., r0 - 1 (compile-time rank
    // indices keep sl[] and the peer pointers in registers)
    const int r0 = (t + d.rank) % d.P;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass)
#pragma unroll
      for (int r = 0; r < LB_EP_MAX_RANKS; ++r)
        if ((pass == 0) == (r >= r0) && sl[r] >= 0) {
          uint4* dst = reinterpret_cast<uint4*>(d.peers.p[r] + d.off_x) +
                       ((long long)d.rank * d.C + sl[r]) * nvec + lane;
#pragma unroll
          for (int u = 0; u < MAXS; ++u)
            if (u < stripes) dst[u * 32] = v[u];
        }
    if (lane < d.k) {
      const int32_t id = d.ids[(long long)t * d.k + lane];
      const float w = d.wf[(long long)t * d.k + lane];
#pragma unroll
      for (int r = 0; r < LB_EP_MAX_RANKS; ++r)
        if (sl[r] >= 0) {
          const long long e = ((long long)d.rank * d.C + sl[r]) * d.k + lane;
          reinterpret_cast<int32_t*>(d.peers.p[r] + d.off_ids)[e] = id;
          reinterpret_cast<float*>(d.peers.p[r] + d.off_w)[e] = w;
        }
    }
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int s_last;
  int* hdr = reinterpret_cast<int*>(d.peers.p[d.rank]);
  if (threadIdx.x == 0) s_last = atomicAdd(hdr + EPH_DONE_DISP, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence_system();
    const int epoch = hdr[EPH_EPOCH] + 1;
    hdr[EPH_EPOCH] = epoch;
    hdr[EPH_DONE_DISP] = 0;
    for (int r = 0; r < d.P; ++r)
      reinterpret_cast<int*>(d.peers.p[r])[EPH_COUNT + d.rank] = d.send_count[r];
    __threadfence_system();
    for (int r = 0; r < d.P; ++r)
      st_release_sys(reinterpret_cast<int*>(d.peers.p[r]) + EPH_DISP + d.rank, epoch);
  }
}

// ------------------------------------------------------------------------------ owner
// Waits for every source's dispatch of this call, then marks the unused rows of each
// recv region (past that source's count) as routed nowhere and, with a placement table,
// turns the received global expert ids into slots (this rank's experts are then the slots
// [rank * E/P, (rank + 1) * E/P), the range the grouped GEMMs select).
__global__ void __launch_bounds__(256) k_ep_recv_prepare(int* hdr, int32_t* __restrict__ recv_ids,
                                                         int P, int C, int k, int E,
                                                         const int32_t* __restrict__ expert_slot,
                                                         int* status) {
  pdl_entry();
  __shared__ int s_cnt[LB_EP_MAX_RANKS];
  if ((int)threadIdx.x < P) {
    const int epoch = hdr[EPH_EPOCH];
    peer_wait(hdr + EPH_DISP + threadIdx.x, epoch, status);
    int c = ld_acquire_sys(hdr + EPH_COUNT + threadIdx.x);
    if (c < 0 || c > C) {
      report(status, LB_DEV_BAD_INDEX);
      c = max(0, min(c, C));
    }
    s_cnt[threadIdx.x] = c;
  }
  __syncthreads();
  const long long n = (long long)P * C * k;
  for (long long f = (long long)blockIdx.x * blockDim.x + threadIdx.x; f < n;
       f += (long long)gridDim.x * blockDim.x) {
    const long long row = f / k;
    const int s = (int)(row / C), i = (int)(row - (long long)s * C);
    if (i >= s_cnt[s]) {
      recv_ids[f] = -1;
    } else if (expert_slot) {
      const int e = recv_ids[f];
      recv_ids[f] = (e >= 0 && e < E) ? expert_slot[e] : -1;
    }
  }
}

struct EpReturn {
  const __nv_bfloat16* yw;
  const int32_t* row_of;
  int H, k, P, C, rank;
  unsigned long long off_ret;
  EpPeers peers;
  int* status;
};

// One warp per received row: the sum of its local experts' weighted rows (fp32, one bf16
// rounding) is written to the source's ret region, slot = the row's position in the
// source's region.  Warp q takes row q / P of source (q + rank) % P, so consecutive warps
// write to different GPUs (a source-major walk would have every GPU storing into the same
// source at the same time).  The last CTA publishes the epoch to every source.
template <int MAXS>  // H <= MAXS * 256
__global__ void __launch_bounds__(256) k_ep_return(const EpReturn d) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x / 32;
  int* hdr = reinterpret_cast<int*>(d.peers.p[d.rank]);
  const int stripes = d.H / 256;
  const int nrows = d.P * d.C;
  for (int q = blockIdx.x * wpb + (int)(threadIdx.x >> 5); q < nrows; q += gridDim.x * wpb) {
    const int s = (q + d.rank) % d.P, i = q / d.P;
    if (i >= min(*(volatile int*)(hdr + EPH_COUNT + s), d.C)) continue;
    const long long rr = (long long)s * d.C + i;   // the row in this rank's recv regions
    const int my_row = lane < d.k ? d.row_of[rr * d.k + lane] : -1;
    float acc[MAXS][8];
#pragma unroll
    for (int u = 0; u < MAXS; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
    for (int j = 0; j < d.k; ++j) {
      const int r = __shfl_sync(0xffffffffu, my_row, j);
      if (r < 0) continue;
      const uint4* src = reinterpret_cast<const uint4*>(d.yw + (long long)r * d.H) + lane;
      uint4 v[MAXS];
#pragma unroll
      for (int u = 0; u < MAXS; ++u)
        if (u < stripes) v[u] = src[u * 32];
#pragma unroll
      for (int u = 0; u < MAXS; ++u)
        if (u < stripes) {
          acc[u][0] += bf16_lo(v[u].x); acc[u][1] += bf16_hi(v[u].x);
          acc[u][2] += bf16_lo(v[u].y); acc[u][3] += bf16_hi(v[u].y);
          acc[u][4] += bf16_lo(v[u].z); acc[u][5] += bf16_hi(v[u].z);
          acc[u][6] += bf16_lo(v[u].w); acc[u][7] += bf16_hi(v[u].w);
        }
    }
    uint8_t* peer = nullptr;
#pragma unroll
    for (int q = 0; q < LB_EP_MAX_RANKS; ++q)
      if (q == s) peer = d.peers.p[q];
    uint4* dst = reinterpret_cast<uint4*>(peer + d.off_ret) +
                 ((long long)d.rank * d.C + i) * (d.H / 8) + lane;
#pragma unroll
    for (int u = 0; u < MAXS; ++u)
      if (u < stripes)
        dst[u * 32] = make_uint4(pack_bf16x2(acc[u][0], acc[u][1]), pack_bf16x2(acc[u][2], acc[u][3]),
                                 pack_bf16x2(acc[u][4], acc[u][5]), pack_bf16x2(acc[u][6], acc[u][7]));
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) s_last = atomicAdd(hdr + EPH_DONE_RET, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence_system();
    const int epoch = hdr[EPH_EPOCH];
    hdr[EPH_DONE_RET] = 0;
    for (int s = 0; s < d.P; ++s)
      st_release_sys(reinterpret_cast<int*>(d.peers.p[s]) + EPH_RET + d.rank, epoch);
  }
}

// ------------------------------------------------------------------------------ combine
// Waits for every owner's return of this call; out[t] = shared row t + the returned rows
// of token t (one per rank it was sent to), fp32 sum, one warp per token.
template <int MAXS>
__global__ void __launch_bounds__(256) k_ep_combine(const __nv_bfloat16* __restrict__ ysh,
                                                    const int32_t* __restrict__ slot, int T,
                                                    int H, int P, int C, int* hdr,
                                                    const __nv_bfloat16* ret, int* status,
                                                    __nv_bfloat16* __restrict__ out) {
  pdl_entry();
  if ((int)threadIdx.x < P) peer_wait(hdr + EPH_RET + threadIdx.x, hdr[EPH_EPOCH], status);
  __syncthreads();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  const int stripes = H / 256;
  float acc[MAXS][8];
#pragma unroll
  for (int u = 0; u < MAXS; ++u)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
  for (int r = -1; r < P; ++r) {
    const __nv_bfloat16* base;
    if (r < 0) {
      base = ysh + (long long)t * H;
    } else {
      const int sl = slot[(long long)t * P + r];
      if (sl < 0) continue;
      base = ret + ((long long)r * C + sl) * H;
    }
    const uint4* src = reinterpret_cast<const uint4*>(base) + lane;
    uint4 v[MAXS];
#pragma unroll
    for (int u = 0; u < MAXS; ++u)
      if (u < stripes) v[u] = src[u * 32];
#pragma unroll
    for (int u = 0; u < MAXS; ++u)
      if (u < stripes) {
        acc[u][0] += bf16_lo(v[u].x); acc[u][1] += bf16_hi(v[u].x);
        acc[u][2] += bf16_lo(v[u].y); acc[u][3] += bf16_hi(v[u].y);
        acc[u][4] += bf16_lo(v[u].z); acc[u][5] += bf16_hi(v[u].z);
        acc[u][6] += bf16_lo(v[u].w); acc[u][7] += bf16_hi(v[u].w);
      }
  }
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * H) + lane;
#pragma unroll
  for (int u = 0; u < MAXS; ++u)
    if (u < stripes)
      dst[u * 32] = make_uint4(pack_bf16x2(acc[u][0], acc[u][1]), pack_bf16x2(acc[u][2], acc[u][3]),
                               pack_bf16x2(acc[u][4], acc[u][5]), pack_bf16x2(acc[u][6], acc[u][7]));
}

// ------------------------------------------------------------------------------ host
struct EpWs {
  MoeWs m;
  int32_t* slot;
  int* send_count;
  uint8_t* mask;      // [C] destination ranks of every token (bit r)
};

static size_t carve_ep(const LbEpArgs& a, void* base, EpWs& w) {
  const size_t C = a.capacity, P = a.world, k = a.top_k, H = a.hidden, E = a.num_experts;
  Carve c(base, ~size_t(0));
  w.m.status = c.take<int>(64);
  w.m.logits = c.take<__nv_bfloat16>(C * E);
  w.m.ids = c.take<int32_t>(C * k);
  w.m.wf = c.take<float>(C * k);
  w.m.wb = c.take<__nv_bfloat16>(C * k);
  w.slot = c.take<int32_t>(C * P);
  w.send_count = c.take<int>(LB_EP_MAX_RANKS);
  w.mask = c.take<uint8_t>(C);
  carve_core(c, C, P * C, k, H, E / P, a.inter, w.m);
  return c.off + 256;
}

static int check_ep(const LbEpArgs* a) {
  LB_REQUIRE(a != nullptr, "lb_ep: null args");
  LB_REQUIRE(a->world >= 1 && a->world <= LB_EP_MAX_RANKS && a->rank >= 0 && a->rank < a->world,
             "lb_ep: need 1 <= world <= %d and 0 <= rank < world", LB_EP_MAX_RANKS);
  LB_REQUIRE(a->capacity > 0 && a->num_tokens >= 0 && a->num_tokens <= a->capacity,
             "lb_ep: need 0 <= num_tokens <= capacity");
  LB_REQUIRE(a->hidden > 0 && a->hidden % 256 == 0 && a->hidden <= 8192,
             "lb_ep: hidden must be a positive multiple of 256 (<= 8192)");
  LB_REQUIRE(a->num_experts > 0 && a->num_experts <= 1024 && a->num_experts % 32 == 0 &&
                 a->num_experts % a->world == 0,
             "lb_ep: num_experts must be a multiple of 32 and of world (<= 1024)");
  LB_REQUIRE(a->top_k > 0 && a->top_k <= 32 && a->top_k <= a->num_experts,
             "lb_ep: top_k in [1, min(32, E)]");
  LB_REQUIRE(a->inter > 0 && a->inter % 128 == 0, "lb_ep: inter must be a multiple of 128");
  LB_REQUIRE(a->capacity * a->world * a->top_k < (1ll << 30), "lb_ep: capacity too large");
  LB_REQUIRE((a->num_tokens == 0 || (a->x && a->out)) && a->w_router && a->w_gate_up &&
                 a->w_down && a->w_shared_gate && a->w_shared_up && a->w_shared_down &&
                 a->w_shared_expert_gate,
             "lb_ep: null tensor");
  for (int r = 0; r < a->world; ++r)
    LB_REQUIRE(a->peer_bufs[r] != nullptr && (reinterpret_cast<uintptr_t>(a->peer_bufs[r]) & 255) == 0,
               "lb_ep: peer buffer %d missing or not 256-byte aligned", r);
  const void* ptrs[] = {a->x, a->out, a->w_router, a->w_gate_up, a->w_down, a->w_shared_gate,
                        a->w_shared_up, a->w_shared_down, a->w_shared_expert_gate};
  for (const void* q : ptrs) LB_REQUIRE(aligned16(q), "lb_ep: tensors must be 16-byte aligned");
  LB_REQUIRE((a->phases & ~7) == 0, "lb_ep: unknown phase bits");
  return LB_OK;
}

}  // namespace lb

using namespace lb;

extern "C" {

size_t lb_ep_buffer_size(int64_t world, int64_t capacity, int64_t hidden, int64_t top_k) {
  if (world < 1 || capacity < 0 || hidden < 0 || top_k < 0) return 0;
  return ep_layout((size_t)world, (size_t)capacity, (size_t)hidden, (size_t)top_k).total;
}

int lb_ep_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == LB_EP_IPC_HANDLE_BYTES, "IPC handle size");
  LB_REQUIRE(ptr && ipc_handle && bytes >= EP_HEADER_BYTES, "lb_ep_buffer_alloc: bad arguments");
  void* p = nullptr;
  LB_CUDA_CHECK(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(LB_ERR_CUDA, "lb_ep_buffer_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return LB_OK;
}

int lb_ep_buffer_open(const void* ipc_handle, void** ptr) {
  LB_REQUIRE(ptr && ipc_handle, "lb_ep_buffer_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  LB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return LB_OK;
}

int lb_ep_buffer_close(void* ptr) {
  LB_REQUIRE(ptr != nullptr, "lb_ep_buffer_close: null pointer");
  LB_CUDA_CHECK(cudaIpcCloseMemHandle(ptr));
  return LB_OK;
}

int lb_ep_buffer_free(void* ptr) {
  LB_REQUIRE(ptr != nullptr, "lb_ep_buffer_free: null pointer");
  LB_CUDA_CHECK(cudaFree(ptr));
  return LB_OK;
}

int lb_ep_workspace_size(const LbEpArgs* a, size_t* bytes) {
  int rc = check_ep(a);
  if (rc) return rc;
  LB_REQUIRE(bytes != nullptr, "lb_ep_workspace_size: null output");
  EpWs w;
  *bytes = carve_ep(*a, nullptr, w);
  return LB_OK;
}

int lb_ep_moe_forward(const LbEpArgs* a, void* stream) {
  int rc = check_ep(a);
  if (rc) return rc;
  EpWs w;
  const size_t need = carve_ep(*a, a->workspace, w);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(LB_ERR_WORKSPACE, "lb_ep_moe_forward: workspace %zu < %zu bytes",
                (size_t)a->workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = (int)a->num_tokens, C = (int)a->capacity, H = (int)a->hidden;
  const int E = (int)a->num_experts, k = (int)a->top_k, I = (int)a->inter;
  const int P = a->world, rank = a->rank, epr = E / P;
  const int phases = a->phases ? a->phases : 7;
  const EpLayout L = ep_layout(P, C, H, k);
  EpPeers peers{};
  for (int r = 0; r < P; ++r) peers.p[r] = static_cast<uint8_t*>(a->peer_bufs[r]);
  uint8_t* own = peers.p[rank];
  int* hdr = reinterpret_cast<int*>(own);
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a->x);
  const int nsm = num_sms();

  if (phases & LB_EP_PHASE_DISPATCH) {
    record_event(a->timing_events[0], st);
    if (T > 0) {
      rc = lb_gemm_bf16(a->x, H, a->w_router, H, w.m.logits, E, T, E, H, 0, 1, w.m.status, stream);
      if (rc) return rc;
      // the shared-expert gate lands in perm_w[0:T), the scale of the shared rows
      rc = launch_topk(w.m.logits, E, T, E, k, w.m.ids, w.m.wf, w.m.wb, x,
                       static_cast<const __nv_bfloat16*>(a->w_shared_expert_gate), H, w.m.perm_w, st);
      if (rc) return rc;
    }
    if (T > 0) {
      launch_k(k_ep_mask, (T * 32 + 255) / 256, 256, 0, st, w.m.ids, T, k, epr, P,
               a->expert_slot, w.mask, w.m.status);
      if ((rc = launched("k_ep_mask"))) return rc;
    }
    launch_k(k_ep_route, 1, 1024, 0, st, w.mask, T, P, w.slot, w.send_count);
    if ((rc = launched("k_ep_route"))) return rc;
    EpDispatch d;
    d.x = x;
    d.ids = w.m.ids;
    d.wf = w.m.wf;
    d.slot = w.slot;
    d.send_count = w.send_count;
    d.T = T;
    d.H = H;
    d.k = k;
    d.P = P;
    d.C = C;
    d.rank = rank;
    d.off_x = L.x;
    d.off_ids = L.ids;
    d.off_w = L.w;
    d.peers = peers;
    d.status = w.m.status;
    const int grid = std::max(1, std::min(nsm * 4, (T + 7) / 8));
    if (H <= 2048)
      launch_k(k_ep_dispatch<8>, grid, 256, 0, st, d);
    else if (H <= 4096)
      launch_k(k_ep_dispatch<16>, grid, 256, 0, st, d);
    else
      launch_k(k_ep_dispatch<32>, grid, 256, 0, st, d);
    if ((rc = launched("k_ep_dispatch"))) return rc;
    record_event(a->timing_events[1], st);
  }

  if (phases & LB_EP_PHASE_EXPERTS) {
    int32_t* recv_ids = reinterpret_cast<int32_t*>(own + L.ids);
    {
      const long long n = (long long)P * C * k;
      const int grid = (int)std::max<long long>(1, std::min<long long>(nsm, (n + 255) / 256));
      launch_k(k_ep_recv_prepare, grid, 256, 0, st, hdr, recv_ids, P, C, k, E, a->expert_slot,
               w.m.status);
      if ((rc = launched("k_ep_recv_prepare"))) return rc;
    }
    MoeCore c{};
    c.T_sh = T;
    c.T_r = P * C;
    c.H = H;
    c.k = k;
    c.I = I;
    c.nl = epr;
    c.expert_base = rank * epr;
    c.x_sh = x;
    c.x_r = reinterpret_cast<const __nv_bfloat16*>(own + L.x);
    c.ids = recv_ids;
    c.wf = reinterpret_cast<const float*>(own + L.w);
    c.w_gate_up = a->w_gate_up;
    c.w_down = a->w_down;
    c.w_sh_gate = a->w_shared_gate;
    c.w_sh_up = a->w_shared_up;
    c.w_sh_down = a->w_shared_down;
    // moe_core records [0],[1] around the gate/up GEMM and [2],[3] around the down GEMM:
    // the caller's events [2] and [3] bracket both
    void* const core_ev[4] = {a->timing_events[2], nullptr, nullptr, a->timing_events[3]};
    c.events = core_ev;
    if ((rc = moe_core(c, w.m, st))) return rc;
    EpReturn d;
    // routed rows follow the T shared-expert rows in yw; row_of indexes all packed rows
    d.yw = w.m.yw;
    d.row_of = w.m.row_of;
    d.H = H;
    d.k = k;
    d.P = P;
    d.C = C;
    d.rank = rank;
    d.off_ret = L.ret;
    d.peers = peers;
    d.status = w.m.status;
    const int grid = std::max(1, std::min(nsm * 4, (P * C + 7) / 8));
    if (H <= 2048)
      launch_k(k_ep_return<8>, grid, 256, 0, st, d);
    else if (H <= 4096)
      launch_k(k_ep_return<16>, grid, 256, 0, st, d);
    else
      launch_k(k_ep_return<32>, grid, 256, 0, st, d);
    if ((rc = launched("k_ep_return"))) return rc;
  }

  if (phases & LB_EP_PHASE_COMBINE) {
    const int blocks = std::max(1, (T * 32 + 255) / 256);
    const __nv_bfloat16* ret = reinterpret_cast<const __nv_bfloat16*>(own + L.ret);
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a->out);
    if (H <= 2048)
      launch_k(k_ep_combine<8>, blocks, 256, 0, st, w.m.yw, w.slot, T, H, P, C, hdr, ret, w.m.status, out);
    else if (H <= 4096)
      launch_k(k_ep_combine<16>, blocks, 256, 0, st, w.m.yw, w.slot, T, H, P, C, hdr, ret, w.m.status, out);
    else
      launch_k(k_ep_combine<32>, blocks, 256, 0, st, w.m.yw, w.slot, T, H, P, C, hdr, ret, w.m.status, out);
    if ((rc = launched("k_ep_combine"))) return rc;
  }
  return LB_OK;
}

}  // extern "C"
