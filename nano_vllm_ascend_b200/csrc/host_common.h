// Host-side helpers shared by the C-ABI entry points: thread-local error
// messages, CUDA error mapping and TMA tensor-map construction.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <utility>

#include "../../include/nvk_paged_kv.h"

namespace nvk {

// Records a message for nvk_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps a CUDA runtime error (if any) to NVK_ERR_CUDA with a message.
int check_cuda(cudaError_t err, const char* what);

// Builds (or fetches from a small cache) a 3-D bf16 TMA tensor map over a
// row-major array [rows, mid, 128] (dims innermost first: {128, mid, rows}),
// box {64, box_mid, box_rows}, 128-byte swizzle. Used for the KV pool
// ([slots, kv_heads, head_dim]), contiguous K/V and queries
// ([tokens, heads, head_dim]). The row stride is mid * 128 elements unless
// row_stride_elems > 0. Returns NVK_OK or an error code.
int kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int mid, int box_rows,
                  int64_t row_stride_elems = 0, int box_mid = 1);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nvk

namespace nvk {
// Raises the kernel's dynamic shared-memory limit to `bytes` on the current
// device (once per kernel and device).
int ensure_dynamic_smem(const void* kernel, size_t bytes);
}  // namespace nvk

namespace nvk {
// Launches `kernel` on `stream` with programmatic stream serialisation, so
// that its prologue (up to pdl_wait()) overlaps the tail of the previous
// kernel in the stream. Inside stream capture this records a programmatic
// graph edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace nvk
