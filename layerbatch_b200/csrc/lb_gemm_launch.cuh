// Host-side launchers of the tcgen05 GEMM kernel templates (dense and grouped expert).
#pragma once

#include "lb_gemm.cuh"
#include "lb_gemm_tok.cuh"
#include "lb_host.h"

#include <algorithm>
#include <atomic>

namespace lb {

template <int BN, int STAGES, int EPI>
int launch_gemm(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& a, int grid,
                cudaStream_t st) {
  auto kern = k_gemm<BN, STAGES, EPI>;
  const size_t smem = GemmSmem<BN, STAGES>::bytes() + (EPI == EPI_F32_PEER ? EPI_STAGE_BYTES : 0);
  if ((int)smem > max_smem_optin())
    return fail(LB_ERR_UNSUPPORTED, "gemm: %zu bytes of shared memory exceed the limit", smem);
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)smem)) return rc;
  if (grid <= 0) return LB_OK;
  launch_k(kern, grid, GEMM_THREADS, smem, st, tA, tB, a);
  { int _rc = launched("k_gemm"); if (_rc) return _rc; }
  return LB_OK;
}

template <int TN, int NBUF, int STAGES, int EPI, int EPW>
int launch_gemm_tok(const CUtensorMap& tW, const CUtensorMap& tWsh0, const CUtensorMap& tWsh1,
                    const CUtensorMap& tX, const CUtensorMap& tXsh, const TokArgs& a, int grid,
                    cudaStream_t st) {
  auto kern = k_gemm_tok<TN, NBUF, STAGES, EPI, EPW>;
  const size_t smem = TokSmem<TN, NBUF, STAGES>::bytes(a.num_groups);
  if ((int)smem > max_smem_optin())
    return fail(LB_ERR_UNSUPPORTED, "gemm_tok: %zu bytes of shared memory exceed the limit", smem);
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)smem)) return rc;
  if (grid <= 0) return LB_OK;
  launch_k(kern, grid, 64 + 32 * EPW, smem, st, tW, tWsh0, tWsh1, tX, tXsh, a);
  { int _rc = launched("k_gemm_tok"); if (_rc) return _rc; }
  return LB_OK;
}

// CTA-pair GEMM (k_gemm_pair): clusters of two CTAs, the persistent grid as many
// clusters as fit the GPU at once (cudaOccupancyMaxActiveClusters, looked up once per
// device), at most one per 256 x 256 tile.
template <int STAGES, int EPI, int EPW>
int launch_gemm_pair(const CUtensorMap& tA, const CUtensorMap& tB, const GemmArgs& a,
                     long long tiles, cudaStream_t st) {
  auto kern = k_gemm_pair<STAGES, EPI, EPW>;
  const size_t smem = PairSmem<STAGES>::bytes();
  if ((int)smem > max_smem_optin())
    return fail(LB_ERR_UNSUPPORTED, "gemm pair: %zu bytes of shared memory exceed the limit", smem);
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)smem)) return rc;
  if (tiles <= 0) return LB_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(64 + 32 * EPW);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::atomic<int> s_clusters[64];
  int dev = 0;
  LB_CUDA_CHECK(cudaGetDevice(&dev));
  int ncl = (dev >= 0 && dev < 64) ? s_clusters[dev].load() : 0;
  if (ncl <= 0) {
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    if (cudaOccupancyMaxActiveClusters(&ncl, kern, &cfg) != cudaSuccess || ncl <= 0) {
      (void)cudaGetLastError();
      ncl = num_sms() / 2;
    }
    if (dev >= 0 && dev < 64) s_clusters[dev].store(ncl);
  }
  cfg.gridDim = dim3(2 * (unsigned)std::min<long long>(tiles, ncl));
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  (void)cudaLaunchKernelEx(&cfg, kern, tA, tB, a);
  { int _rc = launched("k_gemm_pair"); if (_rc) return _rc; }
  return LB_OK;
}

inline GemmArgs gemm_args_default(int* status) {
  GemmArgs a{};
  a.status = status;
  a.splits = 1;
  return a;
}

}  // namespace lb
