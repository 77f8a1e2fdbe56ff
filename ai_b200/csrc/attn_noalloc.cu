// Allocation-free variant of the T = 1 decode attention step (aib_rope_attn_decode_noalloc).
//
// Why it exists: some callers are not allowed to allocate device memory once they are running -- e.g. a
// host application that embeds this library and budgets all device memory itself at start-up (often
// handing everything that is left to the KV cache), or a serving loop that must never enter
// cudaMalloc/cudaFree because those calls can block on, or synchronise with, the whole device. Such a
// caller still owns its inputs and outputs but cannot provide the scratch workspace that
// aib_rope_attn_decode needs. This entry point keeps that scratch in a fixed array of device memory
// belonging to the library instead.
//
// The scratch is `g_attn_noalloc_scratch` below: kNoallocScratchBytes (2 MiB) that every GPU which loads
// the library holds until the process exits. In host code that name is only a host-side stand-in for the
// device symbol, never a device address, so the host looks the real address up with
// cudaGetSymbolAddress -- once per device, with that device current, on the first call made on it (make
// that first call before any stream capture). Every call on a device shares the same array and it keeps
// the last call's contents: the ticket counters are cleared by each call, and calls that could overlap on
// the GPU (two streams, two threads) race on it, so callers must serialise them.
#include <mutex>
#include "common.cuh"

namespace aib {
namespace attn_noalloc {

constexpr size_t kNoallocScratchBytes = 2u << 20;  // 2 MiB per device
constexpr size_t kCounterBytes = 4096;              // ticket counters (up to 1024 KV groups)

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoallocScratchBytes];

// Device address of the scratch array for the current device (looked up once per device).
static int scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(AIB_ECUDA, "aib_rope_attn_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(AIB_ENOTSUP, "aib_rope_attn_decode_noalloc: device index %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return fail(AIB_ECUDA, "aib_rope_attn_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return AIB_OK;
}

}  // namespace attn_noalloc
}  // namespace aib

extern "C" {

int aib_rope_attn_decode_noalloc(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv,
                                 const int64_t* pos, uint16_t* kc, uint16_t* vc, float* out, int H, int KV, int HD,
                                 int maxt, float eps, float scale, void* stream) {
  using namespace aib;
  int rc = attn::check_heads(H, KV, HD);
  if (rc) return rc;
  if (!qkv || !qn || !kn || !inv || !pos || !kc || !vc || !out || maxt <= 0)
    return fail(AIB_EINVAL, "aib_rope_attn_decode_noalloc: bad arguments");
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return fail(AIB_EINVAL, "aib_rope_attn_decode_noalloc: KV caches must be 16-byte aligned");
  const int G = H / KV, S = attn::splits(KV, 1, G, HD);
  const size_t part_bytes = static_cast<size_t>(KV) * S * G * (HD + 2) * sizeof(float);
  if (static_cast<size_t>(KV) * sizeof(int) > attn_noalloc::kCounterBytes ||
      attn_noalloc::kCounterBytes + part_bytes > attn_noalloc::kNoallocScratchBytes)
    return fail(AIB_EINVAL,
                "aib_rope_attn_decode_noalloc: needs %zu bytes of scratch (KV=%d, G=%d, HD=%d, %d splits) but the "
                "fixed scratch holds %zu; use aib_rope_attn_decode with a workspace",
                attn_noalloc::kCounterBytes + part_bytes, KV, G, HD, S, attn_noalloc::kNoallocScratchBytes);
  void* base = nullptr;
  rc = attn_noalloc::scratch_address(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* cnt = static_cast<int*>(base);
  float* part = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + attn_noalloc::kCounterBytes);
  // the counters must start at zero whatever an earlier (possibly interrupted) call left behind
  cudaError_t e = cudaMemsetAsync(cnt, 0, static_cast<size_t>(KV) * sizeof(int), s);
  if (e != cudaSuccess)
    return fail(AIB_ECUDA, "aib_rope_attn_decode_noalloc: clearing counters: %s", cudaGetErrorString(e));
  const size_t smem = HD == 128 ? attn::ring_bytes<128>() : attn::ring_bytes<64>();
  return attn::launch_g<attn::RopeAttnSel>(HD, H / KV, dim3(S, KV), smem, s, "aib_rope_attn_decode_noalloc", qkv, qn,
                                           kn, inv, pos, kc, vc, out, H, KV, maxt, eps, scale, part, cnt,
                                           (H + 2 * KV) * HD, 0LL, H * HD, 0);
}

}  // extern "C"
