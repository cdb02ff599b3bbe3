// The MoE expert stages shared by lb_moe_forward (one GPU) and lb_ep_moe_forward (expert
// parallel): permutation of the routed (row, slot) pairs of the local experts, gather of
// their input rows, the grouped SwiGLU gate/up GEMM and the grouped down GEMM with the
// routing weight fused.  Group 0 of the packed rows is the shared expert (its own input
// rows); groups 1.. are the local experts.
#pragma once

#include <cuda_bf16.h>

#include "lb_host.h"

namespace lb {

struct MoeWs {
  int* status;
  __nv_bfloat16* logits;
  int32_t* ids;
  float* wf;
  __nv_bfloat16* wb;
  int* chunk_hist;
  int* counts;
  int* row_start;
  int* mtile_start;
  int32_t* perm_token;
  float* perm_w;     // [0, T_sh): shared-expert gate; then the routed pairs' weights
  int32_t* row_of;   // [T_r * k]: packed row of pair (t, j), -1 if not a local expert
  __nv_bfloat16* a_packed;
  __nv_bfloat16* act;
  __nv_bfloat16* yw;  // [T_sh + pairs, H]: weighted expert outputs, shared rows first
};

// Carves the permutation / GEMM buffers for T_sh shared-expert rows and T_r routed token
// rows of k slots each.
void carve_core(Carve& c, size_t T_sh, size_t T_r, size_t k, size_t H, size_t nl, size_t I,
                MoeWs& w);

struct MoeCore {
  int T_sh;                       // rows of the shared-expert group (0 = none)
  int T_r;                        // routed token rows
  int H, k, I, nl, expert_base;
  const __nv_bfloat16* x_sh;      // [T_sh, H]
  const __nv_bfloat16* x_r;       // [T_r, H]
  const int32_t* ids;             // [T_r, k] global expert ids (others are skipped)
  const float* wf;                // [T_r, k] routing weights
  const void* w_gate_up;          // [nl, 2I, H]
  const void* w_down;             // [nl, H, I]
  const void* w_sh_gate;          // [I, H]
  const void* w_sh_up;            // [I, H]
  const void* w_sh_down;          // [H, I]
  void* const* events;            // 4 optional cudaEvent_t around the two GEMMs
};

// Permute, gather, gate/up GEMM and down GEMM; perm_w[0, T_sh) must already hold the
// shared-expert gate.  Leaves yw and row_of in the workspace.
int moe_core(const MoeCore& c, const MoeWs& w, cudaStream_t st);

// Router top-k kernel launch (softmax over E, top-k, renormalise; optional shared gate).
int launch_topk(const __nv_bfloat16* logits, long long ld, int T, int E, int k, int32_t* ids,
                float* wf, __nv_bfloat16* wb, const __nv_bfloat16* x, const __nv_bfloat16* wsg,
                int H, float* sg, cudaStream_t st);

}  // namespace lb
