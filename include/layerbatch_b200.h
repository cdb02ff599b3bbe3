/* layerbatch_b200: C ABI of the B200-native (sm_100a) LayerBatch hot path.
 *
 * Every entry point takes plain device pointers, element counts / strides and a CUDA
 * stream (as `void*`, a cudaStream_t; NULL = legacy default stream).  Calls are
 * stream-ordered, perform no host synchronisation and no device allocation: scratch comes
 * from a caller-provided workspace whose size the matching *_workspace_size() returns.
 * All tensors are owned by the caller.  bf16 tensors are row-major with the innermost
 * dimension contiguous.  Errors are returned as status codes (never thrown or trapped);
 * lb_get_last_error_string() describes the last failure of the calling thread.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   lb_moe_forward          <- Qwen3_5SparseMoeBlock.forward   nanovllm/models/qwen3_5.py:899-905
 *                              (router :767-774, experts :802-874, shared expert :903,916-917)
 *   lb_router_topk          <- Qwen3_5TopKRouter.forward tail  nanovllm/models/qwen3_5.py:770-774
 *   lb_moe_permute          <- expert dispatch of _forward_sparse nanovllm/models/qwen3_5.py:821-831
 *   lb_gemm_bf16            <- F.linear / RowParallelLinear.forward nanovllm/layers/linear.py:149-159
 *   lb_store_kvcache        <- store_kvcache                    nanovllm/layers/attention.py:71-80
 *   lb_attn_prologue        <- q/k norms, rotary, store_kvcache nanovllm/models/qwen3_5.py:707-736
 *   lb_qkv_prologue_gemm    <- q/k/v projections + the above   nanovllm/models/qwen3_5.py:705-736
 *   lb_pod_attn_oproj       <- pod_fused_attn_gemm / pod_attn_only nanovllm/layers/pod_kernels.py:237-354
 *                              + Attention.forward decode/prefill nanovllm/layers/attention.py:99-226
 *                              + output gate and o_proj         nanovllm/models/qwen3_5.py:739-746
 */
#ifndef LAYERBATCH_B200_H_
#define LAYERBATCH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define LB_OK 0
#define LB_ERR_INVALID_ARG 1 /* shape, stride, alignment or pointer check failed */
#define LB_ERR_UNSUPPORTED 2 /* valid but not implemented shape (message says which) */
#define LB_ERR_WORKSPACE 3   /* workspace missing or smaller than *_workspace_size() */
#define LB_ERR_CUDA 4        /* a CUDA runtime call failed (launch, attribute, ...) */
#define LB_ERR_DEVICE 5      /* a kernel recorded a device status (lb_read_device_status) */

/* Device status values a kernel may record in the workspace status word. */
#define LB_DEV_OK 0
#define LB_DEV_TIMEOUT 1   /* a bounded pipeline wait gave up */
#define LB_DEV_BAD_INDEX 2 /* an out-of-range page / expert index was skipped */

const char* lb_get_last_error_string(void);
int lb_version(void);
/* Total kernels this library has launched in the process (all threads, all devices). */
unsigned long long lb_kernel_launch_count(void);
/* Number of SMs and the sm_XY of the current device (for host-side planning). */
int lb_device_info(int* num_sms, int* sm_version);

/* Synchronously read (and optionally clear) the device status word that kernels of the
 * call using `workspace` report into.  This is the only entry point that synchronises. */
int lb_read_device_status(const void* workspace, int clear, int* status_out);

/* ---------------------------------------------------------------- dense GEMM
 * C[M,N] = A[M,K] . B[N,K]^T   (bf16 in, fp32 accumulate on tcgen05 tensor cores).
 * c_is_fp32 = 0: C is bf16 and written;   splits must be 1.
 * c_is_fp32 = 1: C is fp32 and ACCUMULATED into (C += A.B^T), K split `splits` ways; the
 *                caller zeroes C first when a plain product is wanted.
 * Requirements: K % 64 == 0, N % 32 == 0, lda/ldb/ldc multiples of 8 elements,
 * pointers 16-byte aligned.  `workspace` needs lb_gemm_workspace_size() bytes. */
size_t lb_gemm_workspace_size(void);
int lb_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                 int64_t M, int64_t N, int64_t K, int c_is_fp32, int splits, void* workspace,
                 void* stream);

/* ---------------------------------------------------------------- router top-k
 * From bf16 router logits [T, E] (row stride ld): softmax in fp32, top-k with ties broken
 * towards the lowest expert index, renormalise over the selected k.
 * Outputs ids [T,k] int32 (descending probability), weights_f32 [T,k] (may be NULL),
 * weights_bf16 [T,k] (may be NULL).  E <= 1024, k <= 32, k <= E. */
int lb_router_topk(const void* logits, int64_t ld, int64_t T, int64_t E, int64_t k,
                   int32_t* ids, float* weights_f32, void* weights_bf16, void* stream);

/* ---------------------------------------------------------------- permutation
 * Expert-major permutation of the (token, slot) pairs of ids [T,k] (global expert ids).
 * Groups: group 0 is the shared expert (rows [0,T), token order); group 1+e is local
 * expert e = id - expert_base for 0 <= e < num_local_experts; other ids are dropped.
 * Inside a group, pairs are ordered slot-major then token (the reference's
 * torch.where(expert_mask[e]) order).
 * Outputs: row_start [G+1] (G = num_local_experts + 1), perm_token [T + T*k] (token of
 * each packed row; rows past row_start[G] are untouched), row_of [T*k] (packed row of
 * pair (t,j) or -1).  With T = 0 only row_start is written (ids, perm_token and row_of
 * may be NULL).  workspace: lb_moe_permute_workspace_size(). */
size_t lb_moe_permute_workspace_size(int64_t T, int64_t k, int64_t num_local_experts);
int lb_moe_permute(const int32_t* ids, int64_t T, int64_t k, int64_t expert_base,
                   int64_t num_local_experts, int32_t* row_start, int32_t* perm_token,
                   int32_t* row_of, void* workspace, size_t workspace_bytes, void* stream);

/* The same permutation for callers that cannot allocate device memory (no workspace):
 * a plugin host whose enqueue hook forbids allocation, or a foreign-language binding
 * without a device allocator.  No counterpart in the reference (which allocates with
 * torch inside the MoE module).  Scratch is a fixed 8,464-byte array in the library's
 * static device memory, held by every GPU that loads the library until exit.
 * Limits: num_local_experts <= 1024 and T*k <= 2^20 pairs (larger returns
 * LB_ERR_UNSUPPORTED): without per-chunk scratch every local expert scans all pairs, so
 * the work grows as num_local_experts * T * k and the cap keeps a call in the
 * low-millisecond range.  The first call on each device looks up that array's address
 * (cudaGetSymbolAddress) and caches it for the life of the process; make that first call
 * before any stream capture, and do not use the entry point on a device after
 * cudaDeviceReset (the cached address then names memory that is no longer mapped).  All
 * calls on a device share the array, so calls that overlap on the GPU (different
 * streams, no ordering between them) race. */
int lb_moe_permute_noalloc(const int32_t* ids, int64_t T, int64_t k, int64_t expert_base,
                           int64_t num_local_experts, int32_t* row_start, int32_t* perm_token,
                           int32_t* row_of, void* stream);

/* ---------------------------------------------------------------- MoE block */
typedef struct LbMoeArgs {
  int64_t num_tokens;        /* T */
  int64_t hidden;            /* H (multiple of 64) */
  int64_t num_experts;       /* E, global routed experts (router width) */
  int64_t top_k;             /* k */
  int64_t inter;             /* I, routed expert intermediate (multiple of 128) */
  int64_t shared_inter;      /* Is, shared expert intermediate (must equal I) */
  int64_t expert_base;       /* first global expert id held in w_gate_up / w_down */
  int64_t num_local_experts; /* experts held locally (E on one GPU; 0 allowed only with
                              * routing_given, e.g. a combine-only call) */
  const void* x;             /* [T, H] bf16, row stride H */
  const void* w_router;      /* [E, H] bf16           mlp.gate.weight */
  const void* w_gate_up;     /* [nl, 2I, H] bf16      mlp.experts.gate_up_proj */
  const void* w_down;        /* [nl, H, I] bf16       mlp.experts.down_proj */
  const void* w_shared_gate; /* [Is, H] bf16          mlp.shared_expert.gate_proj.weight */
  const void* w_shared_up;   /* [Is, H] bf16          mlp.shared_expert.up_proj.weight */
  const void* w_shared_down; /* [H, Is] bf16          mlp.shared_expert.down_proj.weight */
  const void* w_shared_expert_gate; /* [1, H] bf16    mlp.shared_expert_gate.weight
                              * (NULL: the shared expert's rows are not gated, scale 1) */
  void* out;                 /* [T, H] bf16 output */
  void* router_logits;       /* optional out [T, E] bf16 */
  int32_t* topk_ids;         /* optional out [T, k] int32 */
  void* topk_weights;        /* optional out [T, k] bf16 */
  void* workspace;
  size_t workspace_bytes;
  /* optional cudaEvent_t handles recorded on the stream around the grouped gate/up GEMM
   * ([0], [1]) and the grouped down GEMM ([2], [3]); NULL entries are skipped */
  void* timing_events[4];
  /* ---- expert-parallel building blocks (all zero/NULL for the plain block) */
  int32_t routing_given;     /* 1: topk_ids [T,k] (global ids) and topk_weights_f32 are
                              * INPUTS; the router is skipped and w_router may be NULL */
  const float* topk_weights_f32; /* [T, k] fp32 routing weights when routing_given */
  int32_t no_shared;         /* 1: no shared expert (its weights may be NULL) */
  const void* pair_rows;     /* optional [*, H] bf16 rows computed elsewhere (other ranks) */
  const int32_t* pair_index; /* [T, k]: row of pair_rows added into out[t], or -1 */
} LbMoeArgs;

int lb_moe_workspace_size(const LbMoeArgs* args, size_t* bytes);
int lb_moe_forward(const LbMoeArgs* args, void* stream);

/* ---------------------------------------------------------------- expert parallel (NVLink)
 * The MoE block with its experts split over the ranks of one node, exchanging token rows
 * over NVLink through peer-mapped memory instead of a host-driven all-to-all.  The
 * reference has no expert parallelism (every rank holds every expert,
 * nanovllm/models/qwen3_5.py:795-800, and each forward runs the full MoE on its own
 * tokens, qwen3_5.py:899-905); the result equals Qwen3_5SparseMoeBlock.forward on this
 * rank's tokens.  Rank r holds experts [r*E/P, (r+1)*E/P) and one exchange buffer that
 * every rank maps.  Per call: router + top-k on the rank's tokens; each token row is
 * written ONCE to every rank owning at least one of its k experts (with its k ids and
 * weights); the owner runs its experts on the rows it received plus the shared expert
 * on its own tokens in one grouped GEMM pair, sums each received row over its local
 * experts and writes that single row back to the source; the source adds the returned
 * rows to its shared-expert row.  Ranks signal each other with epoch flags in the
 * buffers; every wait is bounded (LB_DEV_TIMEOUT in the workspace status word). */
#define LB_EP_MAX_RANKS 8
#define LB_EP_IPC_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer for `world` ranks, up to `capacity` tokens per rank
 * and call, rows of `hidden` bf16 and `top_k` routed experts.  The buffer calls
 * (alloc / open / close / free) are generic: the tensor-parallel o_proj buffers of
 * lb_pod_attn_oproj use them too. */
size_t lb_ep_buffer_size(int64_t world, int64_t capacity, int64_t hidden, int64_t top_k);
/* cudaMalloc + zero a buffer on the current device and export its CUDA IPC handle
 * (LB_EP_IPC_HANDLE_BYTES bytes written to ipc_handle). */
int lb_ep_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another rank's buffer (same node) into this process; lb_ep_buffer_close unmaps it. */
int lb_ep_buffer_open(const void* ipc_handle, void** ptr);
int lb_ep_buffer_close(void* ptr);
int lb_ep_buffer_free(void* ptr);

#define LB_EP_PHASE_DISPATCH 1 /* router, top-k, routing table, row dispatch + signal */
#define LB_EP_PHASE_EXPERTS 2  /* wait, local experts (+ shared), per-row sums sent back */
#define LB_EP_PHASE_COMBINE 4  /* wait, shared row + returned rows -> out */

typedef struct LbEpArgs {
  int64_t num_tokens;        /* T on this rank (<= capacity) */
  int64_t capacity;          /* tokens per rank per call the buffers were sized for */
  int64_t hidden;            /* H (multiple of 256) */
  int64_t num_experts;       /* E (multiple of world and of 32) */
  int64_t top_k;             /* k */
  int64_t inter;             /* I = shared intermediate (multiple of 128) */
  int32_t rank, world;       /* this rank and the EP group size (world <= LB_EP_MAX_RANKS) */
  const void* x;             /* [T, H] bf16 */
  const void* w_router;      /* [E, H] bf16, replicated */
  const void* w_gate_up;     /* [E/P, 2I, H] bf16: this rank's experts */
  const void* w_down;        /* [E/P, H, I] bf16 */
  const void* w_shared_gate; /* [I, H] */
  const void* w_shared_up;   /* [I, H] */
  const void* w_shared_down; /* [H, I] */
  const void* w_shared_expert_gate; /* [1, H] */
  void* out;                 /* [T, H] bf16 */
  void* peer_bufs[LB_EP_MAX_RANKS]; /* every rank's exchange buffer as mapped in this
                                     * process ([rank] = own), from lb_ep_buffer_* */
  void* workspace;
  size_t workspace_bytes;
  int32_t phases;            /* 0 = all; else a mask of LB_EP_PHASE_* (the phases of
                              * one call must run in order; used to run several ranks'
                              * phases interleaved on one device in tests) */
  void* timing_events[4];    /* optional: around the dispatch ([0],[1]) and the expert
                              * GEMMs ([2],[3]) */
  const int32_t* expert_slot; /* optional [E] device array: expert e lives in slot
                               * expert_slot[e] (rank slot / (E/P), local index slot %
                               * (E/P) of that rank's w_gate_up / w_down); NULL = expert e
                               * in slot e (contiguous ranges).  Lets a placement by
                               * popularity balance the ranks' expert load.  Must be a
                               * permutation of [0, E) and the same on every rank. */
} LbEpArgs;

int lb_ep_workspace_size(const LbEpArgs* args, size_t* bytes);
int lb_ep_moe_forward(const LbEpArgs* args, void* stream);

/* ---------------------------------------------------------------- KV cache store
 * k_cache/v_cache[slot] = k/v[i] for slot_mapping[i] != -1, rows of Hkv*D bf16.
 * k, v: [N, Hkv, D] with token stride k_stride / v_stride (elements), heads packed. */
int lb_store_kvcache(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                     void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t N,
                     int64_t num_slots, int64_t row_elems, void* stream);

/* ---------------------------------------------------------------- attention prologue
 * The full-attention prologue after the projections (nanovllm/models/qwen3_5.py:707-736)
 * fused with store_kvcache (nanovllm/layers/attention.py:50-80), one launch, for every
 * token n, query head h and KV head g:
 *   q_out[n,h]  = RoPE(RMSNorm_1pw(q_in[n,h], q_norm_w))
 *   k_cache[s]  = RoPE(RMSNorm_1pw(k_in[n,g], k_norm_w))   s = slot_mapping[n] (-1: skip)
 *   v_cache[s]  = v_in[n,g]
 * RMSNorm_1pw(x, w) = bf16(fp32 x * rsqrt(mean(x^2) + eps) * (1 + w)) (qwen3_5.py:48-55);
 * RoPE rotates the first rotary_dim dims as two halves with the caller's fp32 cache rows
 * [cos | sin] at positions[n] (rotary_embedding.py:5-54) and rounds to bf16.  q_in may be
 * the query half of q_proj's [N, Hq, 2D] output (q_in_stride_head = 2D), which leaves
 * the gate half in place for lb_pod_attn_oproj. */
typedef struct LbPrologueArgs {
  int64_t num_tokens;          /* N */
  int64_t num_q_heads;         /* Hq */
  int64_t num_kv_heads;        /* Hkv */
  int64_t head_dim;            /* D (256) */
  int64_t rotary_dim;          /* rotated dims (multiple of 16, <= D) */
  float eps;
  const void* q_in;            /* bf16, element (n, h, d) at n*q_in_stride_tok + h*q_in_stride_head + d */
  int64_t q_in_stride_tok, q_in_stride_head;
  const void* k_in;            /* [N, Hkv*D] bf16 rows, token stride k_in_stride_tok */
  int64_t k_in_stride_tok;
  const void* v_in;            /* [N, Hkv*D] bf16 */
  int64_t v_in_stride_tok;
  const void* q_norm_w;        /* [D] bf16  self_attn.q_norm.weight */
  const void* k_norm_w;        /* [D] bf16  self_attn.k_norm.weight */
  const float* cos_sin_cache;  /* [max_position, rotary_dim] fp32 (rotary_emb.cos_sin_cache) */
  int64_t max_position;
  const int64_t* positions;    /* [N] */
  const int32_t* slot_mapping; /* [N] */
  void* k_cache;               /* [num_slots, Hkv*D] bf16 (paged cache viewed as rows) */
  void* v_cache;
  int64_t num_slots;
  void* q_out;                 /* bf16 [N, Hq, D] with the strides below */
  int64_t q_out_stride_tok, q_out_stride_head;
  int* status;                 /* optional device status word (LB_DEV_BAD_INDEX) */
} LbPrologueArgs;

int lb_attn_prologue(const LbPrologueArgs* args, void* stream);

/* The q/k/v projections with the prologue in the GEMM's epilogue (the projections of
 * Qwen3_5FullAttention.forward, nanovllm/models/qwen3_5.py:705-713, then the prologue
 * above): one GEMM x[N, K] . w_qkv^T with w_qkv = [q_proj.weight (per head: query D rows,
 * gate D rows); k_proj.weight; v_proj.weight], [(2*Hq + 2*Hkv)*D, K].  Each 256-column
 * tile of the product is one head row: query rows are normalised, rotated and written to
 * q_out, key rows normalised, rotated and stored into k_cache at slot_mapping, value rows
 * stored into v_cache, and only the gate rows are written to qkv_out ([N, ldo], at the
 * columns the plain GEMM would give them, where lb_pod_attn_oproj reads the gate).  The
 * results are bit-identical to lb_gemm_bf16 followed by lb_attn_prologue.  args supplies
 * N (num_tokens), the heads, eps, the norm weights, positions, slots, caches, q_out and
 * status; its q_in / k_in / v_in are not used.  Requires head_dim 256 and rotary_dim 64
 * (else LB_ERR_UNSUPPORTED), K a multiple of 64, 16-byte aligned rows.  workspace: at
 * least lb_gemm_workspace_size() bytes (status word). */
int lb_qkv_prologue_gemm(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw,
                         void* qkv_out, int64_t ldo, int64_t K, const LbPrologueArgs* args,
                         void* workspace, void* stream);

/* ---------------------------------------------------------------- POD attention + o_proj
 * One batch of sequences, prefill chunks and decode steps mixed in any order.
 * Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) which are its last
 * positions out of context_lens[b] tokens already in the paged cache (bottom-right
 * causal).  Output: out[N, hidden] = (attn(q) * sigmoid(gate)).flatten() . W_o^T. */
typedef struct LbPodArgs {
  int64_t num_seqs;           /* B (<= 16000) */
  int64_t num_tokens;         /* N = cu_seqlens_q[B] */
  int64_t max_q_len;          /* upper bound on any sequence's query length */
  int64_t num_q_heads;        /* Hq */
  int64_t num_kv_heads;       /* Hkv (Hq % Hkv == 0, Hq/Hkv <= 16) */
  int64_t head_dim;           /* D (256) */
  int64_t page_size;          /* tokens per KV block (256) */
  int64_t num_pages;          /* blocks in the cache pool */
  int64_t max_pages_per_seq;  /* block_tables row length */
  int64_t hidden;             /* o_proj output width */
  float sm_scale;
  int32_t kv_split_pages;     /* decode split length in pages (0 = automatic) */
  const void* q;              /* [N, Hq, D] bf16 */
  int64_t q_stride_tok, q_stride_head;
  const void* gate;           /* [N, Hq, D] bf16 (pre-sigmoid output gate), NULL = no gate */
  int64_t gate_stride_tok, gate_stride_head;
  const void* k_cache;        /* [num_pages, page_size, Hkv, D] bf16 */
  const void* v_cache;
  const int32_t* block_tables;/* [B, max_pages_per_seq] int32 */
  const int32_t* context_lens;/* [B] int32 */
  const int32_t* cu_seqlens_q;/* [B+1] int32 */
  const void* w_o;            /* [hidden, Hq*D] bf16; NULL = attention only (then attn_out
                               * is required and out / hidden are ignored) */
  void* attn_out;             /* optional out: [N, Hq*D] bf16 attention output (pre-gate) */
  void* out;                  /* [N, hidden] bf16, or fp32 when out_fp32 */
  int32_t out_fp32;           /* 1: write fp32 o_proj partials (tensor-parallel reduce) */
  void* workspace;
  size_t workspace_bytes;
  /* optional cudaEvent_t handles recorded around the attention kernel ([0], [1]) and the
   * o_proj GEMM ([2], [3]); NULL entries are skipped */
  void* timing_events[4];
  /* optional host-side work hints (0 = estimate from the shapes): query-key pairs of the
   * prefill rows (sum over prefill sequences of L*(C-L) + L*(L+1)/2) and context tokens
   * of the decode sequences; they set how many SMs start on prefill tiles */
  int64_t prefill_pairs_hint;
  int64_t decode_tokens_hint;
  /* ---- tensor parallel o_proj (optional; tp_size <= 1 = off).  This rank holds a slice
   * of the heads and W_o's matching columns; the o_proj GEMM stores each fp32 128-row
   * tile of its partial straight into the inbox of the rank that owns the tile (tile m
   * -> rank m % tp_size, NVLink stores), the owner sums the tp_size partials in rank
   * order and sends the bf16 rows to every rank, so `out` (bf16) ends with the
   * all-reduced result on every rank: RowParallelLinear's fp32 all-reduce
   * (nanovllm/layers/linear.py:149-157) fused into the GEMM. */
  int32_t tp_rank, tp_size;
  int64_t tp_capacity;             /* rows the TP buffers were sized for (>= num_tokens) */
  void* tp_bufs[LB_EP_MAX_RANKS];  /* every rank's TP buffer (lb_tp_buffer_size bytes,
                                    * from lb_ep_buffer_alloc / lb_ep_buffer_open) */
  int32_t tp_phases;               /* 0 = all; else a mask of LB_TP_PHASE_* (tests) */
  /* ---- fused attention prologue (optional; NULL = q is final).  The call then runs the
   * prologue of lb_attn_prologue for its num_tokens tokens inside the attention kernel:
   * the CTAs first normalise and rotate every query row into q (which must be the
   * prologue's q_out, same strides) and store every new K/V row into the paged cache (the
   * prologue's k_cache / v_cache, num_slots = num_pages * page_size); each attention item
   * waits (bounded) for its sequence's rows before it loads them.  Replaces the separate
   * lb_attn_prologue launch in front of this call. */
  const LbPrologueArgs* prologue;
} LbPodArgs;

#define LB_TP_PHASE_ATTN 1    /* attention, merge, o_proj GEMM to the owners + signal */
#define LB_TP_PHASE_REDUCE 2  /* wait, sum the owned rows, send them to every rank */
#define LB_TP_PHASE_GATHER 4  /* wait, copy the rows other ranks own into out */

/* Bytes of one rank's tensor-parallel exchange buffer for `world` ranks, up to
 * `capacity` rows of `hidden` outputs. */
size_t lb_tp_buffer_size(int64_t world, int64_t capacity, int64_t hidden);

int lb_pod_workspace_size(const LbPodArgs* args, size_t* bytes);
int lb_pod_attn_oproj(const LbPodArgs* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LAYERBATCH_B200_H_ */
