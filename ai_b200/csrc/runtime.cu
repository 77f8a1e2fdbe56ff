// Library-wide host runtime: error messages, PDL switch, device status word, tensor-map encoding.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <set>
#include <utility>
#include "common.cuh"

namespace aib {
namespace attn {
extern int g_cluster_sizes;  // attn.cu
}
namespace gemv {
extern int g_variant;  // gemv.cu
}

static thread_local char t_err[512] = {0};
static int g_pdl = 1;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

bool pdl_enabled() { return g_pdl != 0; }

int sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 && cudaGetDevice(&device) != cudaSuccess) return 148;
  if (device >= 64) device = 63;
  if (!cache[device]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

bool smem_raised(const void* kernel, int device, bool record) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> seen;
  std::lock_guard<std::mutex> lock(mu);
  if (record) seen.insert({kernel, device});
  return seen.count({kernel, device}) != 0;
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AIB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return AIB_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda dependency)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_map_3d_u8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                   uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AIB_ECUDA, "cuTensorMapEncodeTiled is not available");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (s1_bytes & 15) || (s2_bytes & 15))
    return fail(AIB_EINVAL, "tensor map: base/strides must be 16-byte aligned");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AIB_OK;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, int rank, const void* base,
             const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(AIB_ECUDA, "cuTensorMapEncodeTiled is not available");
  if (rank < 1 || rank > 5) return fail(AIB_EINVAL, "tensor map: rank %d", rank);
  if (reinterpret_cast<uintptr_t>(base) & 15) return fail(AIB_EINVAL, "tensor map: base must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] & 15) return fail(AIB_EINVAL, "tensor map: strides must be multiples of 16 bytes");
  if ((box[0] * static_cast<uint32_t>(elem_bytes)) & 15)
    return fail(AIB_EINVAL, "tensor map: the inner box must be a multiple of 16 bytes");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AIB_OK;
}

}  // namespace aib

extern "C" {

int aib_abi_version(void) { return AIB_ABI_VERSION; }

const char* aib_last_error(void) { return aib::t_err; }

void aib_set_pdl(int enabled) { aib::g_pdl = enabled ? 1 : 0; }

int aib_debug_knob(int knob, int value) {
  cudaError_t e = cudaSuccess;
  if (knob == 1) {
    const uint32_t v = value > 0 ? static_cast<uint32_t>(value) : 0u;
    e = cudaMemcpyToSymbol(aib::g_aib_spin_override, &v, sizeof(v));
  } else if (knob == 2) {
    const int v = value ? 1 : 0;
    e = cudaMemcpyToSymbol(aib::g_aib_withhold_copies, &v, sizeof(v));
  } else if (knob == 3) {
    if (value < 0 || value > 2) return aib::fail(AIB_EINVAL, "aib_debug_knob(3): value %d not in 0..2", value);
    aib::attn::g_cluster_sizes = value;
  } else if (knob == 4) {
    if (value != 1 && value != 3 && value != 4) return aib::fail(AIB_EINVAL, "aib_debug_knob(4): value %d", value);
    aib::gemv::g_variant = value;
  } else {
    return aib::fail(AIB_EINVAL, "aib_debug_knob: unknown knob %d", knob);
  }
  if (e != cudaSuccess) return aib::fail(AIB_ECUDA, "aib_debug_knob: %s", cudaGetErrorString(e));
  return AIB_OK;
}

int aib_status_read(int* out, int clear) {
  if (!out) return aib::fail(AIB_EINVAL, "aib_status_read: out is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(out, aib::g_aib_status, sizeof(int));
  if (e != cudaSuccess) return aib::fail(AIB_ECUDA, "aib_status_read: %s", cudaGetErrorString(e));
  if (clear) {
    int z = 0;
    e = cudaMemcpyToSymbol(aib::g_aib_status, &z, sizeof(int));
    if (e != cudaSuccess) return aib::fail(AIB_ECUDA, "aib_status_read(clear): %s", cudaGetErrorString(e));
  }
  return AIB_OK;
}

}  // extern "C"
