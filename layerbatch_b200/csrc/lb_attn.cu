// Paged attention hot path: KV-cache store, POD attention + gated o_proj.
#include "lb_gemm_launch.cuh"
#include "lb_host.h"

namespace lb {

// One warp per token row: copy k/v rows of `row_elems` bf16 into the slot given by
// slot_mapping (skip -1; out-of-range slots are skipped too).
__global__ void k_store_kvcache(const __nv_bfloat16* __restrict__ k, long long ks,
                                const __nv_bfloat16* __restrict__ v, long long vs,
                                __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                const int32_t* __restrict__ slots, int n, long long num_slots,
                                int row_elems) {
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
  k_store_kvcache<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(k), k_stride, static_cast<const __nv_bfloat16*>(v),
      v_stride, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
      slot_mapping, (int)N, num_slots, (int)row_elems);
  LB_CUDA_CHECK(cudaGetLastError());
  return LB_OK;
}

int lb_pod_workspace_size(const LbPodArgs* a, size_t* bytes) {
  (void)a;
  (void)bytes;
  return fail(LB_ERR_UNSUPPORTED, "lb_pod_workspace_size: not built yet");
}

int lb_pod_attn_oproj(const LbPodArgs* a, void* stream) {
  (void)a;
  (void)stream;
  return fail(LB_ERR_UNSUPPORTED, "lb_pod_attn_oproj: not built yet");
}

}  // extern "C"
