// Peer-memory exchange shared by the tensor-parallel o_proj reduction (lb_attn.cu, the
// GEMM epilogue in lb_gemm.cuh) and expert parallelism (lb_ep.cu): ranks of one node map
// each other's buffers (CUDA IPC) and order their phases with per-call epoch flags.
#pragma once

#include <cstdint>

namespace lb {

constexpr int LB_PEER_MAX = 8;

// Tensor-parallel exchange buffer of one rank: a 4 KiB header, then
//   inbox  [P][cap][H] fp32: rank s's o_proj partial rows owned by this rank (region s)
//   gather [cap][H]    bf16: reduced rows owned by other ranks, written by their owners
// Header ints (each group on its own 128-byte line):
constexpr int TPH_PART = 0;       // [s]: epoch of the partials rank s stored here
constexpr int TPH_GATH = 32;      // [s]: epoch of the reduced rows rank s stored here
constexpr int TPH_EPOCH = 64;     // this rank's call counter (own GPU only)
constexpr int TPH_DONE_GEMM = 96; // CTA completion counters (own GPU only)
constexpr int TPH_DONE_RED = 128;
constexpr unsigned long long TP_HEADER_BYTES = 4096;

// What the o_proj GEMM epilogue needs to send its fp32 tiles to their owners: 128-row
// m-tile m belongs to rank m % size.
struct TpPeers {
  float* inbox[LB_PEER_MAX];  // every rank's inbox as mapped in this process
  int* hdr[LB_PEER_MAX];      // every rank's header
  int rank, size;
  long long inbox_rows;       // cap: rows of one source region
};

}  // namespace lb
