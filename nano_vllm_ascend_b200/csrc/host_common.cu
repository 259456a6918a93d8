// Host-side helpers: error reporting and cached TMA tensor maps.
#include "host_common.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace nvk {

namespace {

thread_local char g_last_error[512] = "";

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver symbol is resolved through the runtime so that the library does
// not link libcuda directly (it loads on hosts without a driver).
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* base;
  int64_t rows;
  int mid;
  int box_rows;
  int64_t row_stride;
  int box_mid;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && mid == o.mid && box_rows == o.box_rows &&
           row_stride == o.row_stride && box_mid == o.box_mid;
  }
};

// Tiny direct-mapped cache: a decode step re-encodes the same 2 maps per
// layer; encoding is cheap but not free on the launch path.
constexpr int kCacheSlots = 256;
struct CacheEntry {
  bool valid = false;
  MapKey key{};
  CUtensorMap map{};
};
CacheEntry g_cache[kCacheSlots];
std::mutex g_cache_mu;

size_t hash_key(const MapKey& k) {
  uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
  h ^= static_cast<uint64_t>(k.rows) + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2);
  h ^= static_cast<uint64_t>(k.mid * 131 + k.box_rows * 7 + k.box_mid) + (h << 6) + (h >> 2);
  h ^= static_cast<uint64_t>(k.row_stride) + (h << 6) + (h >> 2);
  return static_cast<size_t>(h % kCacheSlots);
}

}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return NVK_OK;
  return fail(NVK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int mid, int box_rows,
                  int64_t row_stride_elems, int box_mid) {
  if (row_stride_elems <= 0) row_stride_elems = static_cast<int64_t>(mid) * 128;
  const MapKey key{base, rows, mid, box_rows, row_stride_elems, box_mid};
  const size_t slot = hash_key(key);
  {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (g_cache[slot].valid && g_cache[slot].key == key) {
      *out = g_cache[slot].map;
      return NVK_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(NVK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  if (!aligned16(base)) return fail(NVK_ERR_INVALID_ARGUMENT, "tensor base %p is not 16-byte aligned", base);
  if (rows <= 0 || rows > (int64_t(1) << 31) - 1)
    return fail(NVK_ERR_UNSUPPORTED, "tensor map row count %lld outside TMA range", (long long)rows);
  if ((row_stride_elems * 2) % 16 != 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "row stride %lld elements is not a multiple of 16 bytes",
                (long long)row_stride_elems);
  const cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(mid), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(row_stride_elems) * 2};
  if (box_mid < 1 || box_mid > mid || box_rows < 1 || box_rows > 256)
    return fail(NVK_ERR_INVALID_ARGUMENT, "tensor map box {64, %d, %d} outside {%d, %lld}", box_mid, box_rows, mid,
                (long long)rows);
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_mid), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estride[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NVK_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    g_cache[slot].valid = true;
    g_cache[slot].key = key;
    g_cache[slot].map = map;
  }
  *out = map;
  return NVK_OK;
}

int ensure_dynamic_smem(const void* kernel, size_t bytes) {
  struct Done {
    const void* kernel;
    int device;
    size_t bytes;
  };
  static Done done[64];
  static int ndone = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < ndone; ++i)
    if (done[i].kernel == kernel && done[i].device == dev && done[i].bytes >= bytes) return NVK_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (ndone < 64) done[ndone++] = Done{kernel, dev, bytes};
  return NVK_OK;
}

}  // namespace nvk

extern "C" const char* nvk_last_error(void) { return nvk::g_last_error; }

extern "C" int nvk_abi_version(void) { return 5; }
