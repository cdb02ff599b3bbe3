// Host-side helpers shared by the C-ABI entry points: error reporting, TMA tensor-map
// encoding (through the driver entry point, so the library does not link libcuda), and
// workspace carving.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/layerbatch_b200.h"

namespace lb {

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

// Check a CUDA runtime call; on failure record the error and return LB_ERR_CUDA.
#define LB_CUDA_CHECK(expr)                                                        \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess)                                                         \
      return ::lb::fail(LB_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,               \
                        cudaGetErrorString(_e), __FILE__, __LINE__);               \
  } while (0)

#define LB_REQUIRE(cond, ...)                                                      \
  do {                                                                             \
    if (!(cond)) return ::lb::fail(LB_ERR_INVALID_ARG, __VA_ARGS__);               \
  } while (0)

// 2-D bf16 tensor map: `rows` x `cols` (cols contiguous), row pitch in elements.
int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                      uint64_t row_pitch_elems, uint32_t box_rows, uint32_t box_cols);
// 3-D bf16 tensor map: depth x rows x cols (cols contiguous).
int make_tmap_bf16_3d(CUtensorMap* m, const void* base, uint64_t depth, uint64_t rows,
                      uint64_t cols, uint64_t row_pitch_elems, uint64_t depth_pitch_elems,
                      uint32_t box_rows, uint32_t box_cols);

// General 3-D bf16 tensor map: dims (d2, d1, d0) outermost first, d0 contiguous, strides
// of dims 2 and 1 in elements, box (b2, b1, b0).
int make_tmap_bf16_3d_box(CUtensorMap* m, const void* base, uint64_t d2, uint64_t d1,
                          uint64_t d0, uint64_t s2_elems, uint64_t s1_elems, uint32_t b2,
                          uint32_t b1, uint32_t b0);

// Count one kernel launch of this library and check the launch error.
int launched(const char* what);

// Whether kernels are launched with programmatic stream serialization (programmatic
// dependent launch); on unless the environment sets LB_PDL=0.
bool pdl_enabled();

// Launch `kern` on `st` with the programmatic-serialization attribute (see pdl_entry in
// the device helpers); errors surface through launched().
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
void record_event(void* ev, cudaStream_t st);

int num_sms();
int max_smem_optin();

// Dense bf16 GEMM C = A . B^T with epilogue `epi` (an EpiKind of lb_gemm.cuh); the body of
// lb_gemm_bf16, also used for the library's internal split-K projections.
int gemm_run(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
             int64_t M, int64_t N, int64_t K, int epi, int splits, int* status, cudaStream_t st);

// Raise a kernel's dynamic shared-memory limit on the current device to at least `bytes`.
// The attribute is set once per (kernel, device) and cached, so steady-state calls (and
// calls made while a stream is being captured into a CUDA graph) make no runtime call.
int ensure_smem_attr(const void* func, int bytes);

// Bump allocator over a caller-provided workspace (256-byte aligned sub-buffers).
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t off = 0;
  Carve(void* b, size_t c) : base(static_cast<uint8_t*>(b)), cap(c) {}
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
  bool ok() const { return off <= cap; }
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace lb
