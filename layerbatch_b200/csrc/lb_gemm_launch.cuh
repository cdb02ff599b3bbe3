// Host-side launcher for the grouped tcgen05 GEMM kernel template.
#pragma once

#include "lb_gemm.cuh"
#include "lb_host.h"

namespace lb {

template <int BN, int STAGES, int EPI, bool TWO_HALVES>
int launch_gemm(const CUtensorMap& tA, const CUtensorMap& tAsh, const CUtensorMap& tB,
                const CUtensorMap& tBsh0, const CUtensorMap& tBsh1, const GemmArgs& a,
                int grid, cudaStream_t st) {
  auto kern = k_gemm<BN, STAGES, EPI, TWO_HALVES>;
  const size_t smem = GemmSmem<BN, STAGES>::bytes(a.num_groups) +
                      (EPI == EPI_F32_PEER ? EPI_STAGE_BYTES : 0);
  if ((int)smem > max_smem_optin())
    return fail(LB_ERR_UNSUPPORTED, "gemm: %zu bytes of shared memory exceed the limit", smem);
  if (int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)smem)) return rc;
  if (grid <= 0) return LB_OK;
  launch_k(kern, grid, GEMM_THREADS, smem, st, tA, tAsh, tB, tBsh0, tBsh1, a);
  { int _rc = launched("kern"); if (_rc) return _rc; }
  return LB_OK;
}

inline GemmArgs gemm_args_default(int* status) {
  GemmArgs a{};
  a.status = status;
  a.mtile_start = nullptr;
  a.row_start = nullptr;
  a.num_groups = 1;
  a.splits = 1;
  a.shared_group = -1;
  a.b_group_base = 0;
  a.b_half_offset = 0;
  return a;
}

}  // namespace lb
