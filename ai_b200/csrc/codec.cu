// 12-bit lossless bf16 codec: encoders (host + device) and the exact row decoder.
//
// Format (reference `ramvi/engine/ramvi_engine/kernels/wcomp.py:1-32`): W [N,K] bf16, K % 256 == 0.
//   e = (bits >> 7) & 0xFF; base = first argmax over windows [b, b+14] of the exponent histogram;
//   code = e - base, or 15 when outside 0..14 (an exception); m8 = sign << 7 | mantissa;
//   e4: in each 256-chunk, byte i = code(i) | code(128 + i) << 4;
//   exceptions as CSR: rp [N+1], er/ec row-major, ev = fp32 of the bf16 value.
// Decode (wcomp.py:48-54): fp32 bits = sign << 31 | (code + base) << 23 | mantissa << 16, 0 for code 15,
// then the exception values are scattered in.
#include <algorithm>
#include <cstring>
#include "common.cuh"

namespace aib {
namespace codec {

constexpr int CH = 256;

// ---------------------------------------------------------------------------------- host encoder
static int choose_base(const uint64_t* cnt) {
  uint64_t cs[257];
  cs[0] = 0;
  for (int i = 0; i < 256; ++i) cs[i + 1] = cs[i] + cnt[i];
  int base = 0;
  uint64_t best = 0;
  for (int b = 0; b + 15 <= 256; ++b) {  // windows [b, b+14]; strict '>' keeps the first maximum
    const uint64_t s = cs[b + 15] - cs[b];
    if (b == 0 || s > best) best = s, base = b;
  }
  return base;
}

static int encode_host(const uint16_t* w, int N, int K, uint8_t* m8, uint8_t* e4, int32_t* rp, int32_t* base_out,
                       int64_t* n_exc, int32_t* er, int32_t* ec, float* ev, int64_t cap) {
  if (!w || !m8 || !e4 || !rp || !base_out || !n_exc || N <= 0 || K <= 0 || K % CH)
    return fail(AIB_EINVAL, "aib_c12_encode_host: bad arguments (N=%d K=%d, K must be a positive multiple of 256)",
                N, K);
  const size_t n = static_cast<size_t>(N) * K;
  uint64_t cnt[256] = {0};
  for (size_t i = 0; i < n; ++i) cnt[(w[i] >> 7) & 0xFF]++;
  const int base = choose_base(cnt);
  int64_t ne = 0;
  rp[0] = 0;
  for (int r = 0; r < N; ++r) {
    const uint16_t* row = w + static_cast<size_t>(r) * K;
    for (int c0 = 0; c0 < K; c0 += CH) {
      for (int i = 0; i < CH / 2; ++i) {
        int code[2];
        for (int h = 0; h < 2; ++h) {
          const int k = c0 + h * (CH / 2) + i;
          const uint16_t b = row[k];
          int c = ((b >> 7) & 0xFF) - base;
          if (c < 0 || c > 14) c = 15;
          code[h] = c;
          m8[static_cast<size_t>(r) * K + k] = static_cast<uint8_t>(((b >> 15) << 7) | (b & 0x7F));
        }
        e4[static_cast<size_t>(r) * (K / 2) + c0 / 2 + i] = static_cast<uint8_t>(code[0] | (code[1] << 4));
      }
    }
    for (int k = 0; k < K; ++k) {
      const int c = ((row[k] >> 7) & 0xFF) - base;
      if (c < 0 || c > 14) {
        if (er && ec && ev && ne < cap) {
          er[ne] = r;
          ec[ne] = k;
          const uint32_t u = static_cast<uint32_t>(row[k]) << 16;
          std::memcpy(&ev[ne], &u, 4);
        }
        ++ne;
      }
    }
    if (ne > INT32_MAX) return fail(AIB_EINVAL, "aib_c12_encode_host: more than 2^31 exceptions");
    rp[r + 1] = static_cast<int32_t>(ne);
  }
  *base_out = base;
  *n_exc = ne;
  if (ne > cap || (ne > 0 && (!er || !ec || !ev)))
    return fail(AIB_ESPACE, "aib_c12_encode_host: %lld exceptions, capacity %lld", (long long)ne, (long long)cap);
  return AIB_OK;
}

// -------------------------------------------------------------------------------- device encoder
// Pass 1a: exponent histogram (256 bins, 64-bit counts in the workspace).
__global__ void hist_kernel(const uint16_t* __restrict__ w, size_t n, unsigned long long* __restrict__ gcnt) {
  __shared__ unsigned int h[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const size_t n8 = n / 8;
  const uint4* w8 = reinterpret_cast<const uint4*>(w);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const uint4 v = __ldg(&w8[i]);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      atomicAdd(&h[(u[k] >> 7) & 0xFF], 1u);
      atomicAdd(&h[(u[k] >> 23) & 0xFF], 1u);
    }
  }
  for (size_t i = n8 * 8 + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    atomicAdd(&h[(w[i] >> 7) & 0xFF], 1u);
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (h[i]) atomicAdd(&gcnt[i], static_cast<unsigned long long>(h[i]));
}

// Pass 1b: base = first argmax of the 15-wide window sums.
__global__ void base_kernel(const unsigned long long* __restrict__ gcnt, int32_t* base_out) {
  if (threadIdx.x != 0) return;
  unsigned long long s = 0;  // sliding window sum over [b, b+14]
  for (int i = 0; i < 15; ++i) s += gcnt[i];
  int base = 0;
  unsigned long long best = s;
  for (int b = 1; b + 15 <= 256; ++b) {
    s += gcnt[b + 14] - gcnt[b - 1];
    if (s > best) best = s, base = b;
  }
  *base_out = base;
}

// Pass 1c: planes + per-row exception counts. One block per row, thread per e4 byte.
__global__ void planes_kernel(const uint16_t* __restrict__ w, int N, int K, const int32_t* __restrict__ base_p,
                              uint8_t* __restrict__ m8, uint8_t* __restrict__ e4, int32_t* __restrict__ rowcnt) {
  const int r = blockIdx.x;
  if (r >= N) return;
  const int base = *base_p;
  const uint16_t* row = w + static_cast<size_t>(r) * K;
  int cnt = 0;
  for (int b = threadIdx.x; b < K / 2; b += blockDim.x) {
    const int c0 = (b / (CH / 2)) * CH, i = b % (CH / 2);
    int code[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = c0 + h * (CH / 2) + i;
      const uint16_t v = row[k];
      int c = ((v >> 7) & 0xFF) - base;
      if (c < 0 || c > 14) c = 15, ++cnt;
      code[h] = c;
      m8[static_cast<size_t>(r) * K + k] = static_cast<uint8_t>(((v >> 15) << 7) | (v & 0x7F));
    }
    e4[static_cast<size_t>(r) * (K / 2) + b] = static_cast<uint8_t>(code[0] | (code[1] << 4));
  }
  __shared__ int red[32];
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) s += red[i];
    rowcnt[r] = s;
  }
}

// Pass 1d: exclusive scan of the row counts into rp[0..N] (single block, deterministic).
__global__ void scan_kernel(const int32_t* __restrict__ rowcnt, int N, int32_t* __restrict__ rp) {
  __shared__ long long part[1024];
  const int t = threadIdx.x, nt = blockDim.x;
  const int per = (N + nt - 1) / nt;
  const int a = min(N, t * per), b = min(N, a + per);
  long long s = 0;
  for (int i = a; i < b; ++i) s += rowcnt[i];
  part[t] = s;
  __syncthreads();
  if (t == 0) {
    long long run = 0;
    for (int i = 0; i < nt; ++i) {
      const long long v = part[i];
      part[i] = run;
      run += v;
    }
    rp[N] = static_cast<int32_t>(run);
  }
  __syncthreads();
  long long run = part[t];
  for (int i = a; i < b; ++i) {
    rp[i] = static_cast<int32_t>(run);
    run += rowcnt[i];
  }
}

// Pass 2: exception lists, one warp per row, row-major order via ballot compaction.
__global__ void exc_kernel(const uint16_t* __restrict__ w, int N, int K, int base, const int32_t* __restrict__ rp,
                           int32_t* __restrict__ er, int32_t* __restrict__ ec, float* __restrict__ ev) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  const int r = warp;
  int out = rp[r];
  const int end = rp[r + 1];
  if (out == end) return;
  const uint16_t* row = w + static_cast<size_t>(r) * K;
  for (int k0 = 0; k0 < K; k0 += 32) {
    const uint16_t v = row[k0 + lane];
    const int c = ((v >> 7) & 0xFF) - base;
    const bool x = (c < 0 || c > 14);
    const unsigned m = __ballot_sync(0xffffffffu, x);
    if (x) {
      const int o = out + __popc(m & ((1u << lane) - 1u));
      if (o < end) {
        er[o] = r;
        ec[o] = k0 + lane;
        ev[o] = __uint_as_float(static_cast<uint32_t>(v) << 16);
      } else {
        set_status(AIB_DEV_OVERFLOW);
      }
    }
    out += __popc(m);
  }
}

// --------------------------------------------------------------------------------------- decode
// One block per row: decode the planes (code 15 -> 0), then scatter the row's exceptions.
template <int OUT_BF16>
__global__ void decode_kernel(aib_c12 c, int first, int last, void* __restrict__ out) {
  const int r = first + blockIdx.x;
  pdl_wait();
  if (r >= last) return;
  const int K = c.K;
  const uint8_t* m8 = c.m8 + static_cast<size_t>(r) * K;
  const uint8_t* e4 = c.e4 + static_cast<size_t>(r) * (K / 2);
  const size_t o = static_cast<size_t>(blockIdx.x) * K;
  for (int b = threadIdx.x; b < K / 2; b += blockDim.x) {
    const int c0 = (b / (CH / 2)) * CH, i = b % (CH / 2);
    const uint32_t e = e4[b];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = c0 + h * (CH / 2) + i;
      const uint32_t code = h ? (e >> 4) : (e & 15u);
      const uint32_t m = m8[k];
      uint32_t bits = ((m & 0x80u) << 24) | ((code + static_cast<uint32_t>(c.base)) << 23) | ((m & 0x7Fu) << 16);
      if (code == 15u) bits = 0;
      if (OUT_BF16)
        static_cast<uint16_t*>(out)[o + k] = static_cast<uint16_t>(bits >> 16);
      else
        static_cast<float*>(out)[o + k] = __uint_as_float(bits);
    }
  }
  __syncthreads();
  const int a = c.rp[r], z = c.rp[r + 1];
  for (int j = a + threadIdx.x; j < z; j += blockDim.x) {
    const int col = c.ec[j];
    if (col < 0 || col >= K) {
      set_status(AIB_DEV_OVERFLOW);
      continue;
    }
    const float v = c.ev[j];
    if (OUT_BF16)
      static_cast<uint16_t*>(out)[o + col] = static_cast<uint16_t>(__float_as_uint(v) >> 16);
    else
      static_cast<float*>(out)[o + col] = v;
  }
  pdl_trigger();
}

}  // namespace codec
}  // namespace aib

using namespace aib;

extern "C" {

int aib_c12_encode_host(const uint16_t* w, int N, int K, uint8_t* m8, uint8_t* e4, int32_t* rp, int32_t* base,
                        int64_t* n_exc, int32_t* er, int32_t* ec, float* ev, int64_t exc_cap) {
  return codec::encode_host(w, N, K, m8, e4, rp, base, n_exc, er, ec, ev, exc_cap);
}

size_t aib_c12_encode_workspace(int N) {
  return 256 * sizeof(unsigned long long) + (N > 0 ? static_cast<size_t>(N) : 0) * sizeof(int32_t);
}

int aib_c12_encode_planes(const uint16_t* w, int N, int K, uint8_t* m8, uint8_t* e4, int32_t* rp, int32_t* base_out,
                          void* ws, size_t ws_bytes, void* stream) {
  if (!w || !m8 || !e4 || !rp || !base_out || N <= 0 || K <= 0 || K % codec::CH)
    return fail(AIB_EINVAL, "aib_c12_encode_planes: bad arguments (N=%d K=%d)", N, K);
  if (!ws || ws_bytes < aib_c12_encode_workspace(N))
    return fail(AIB_EWORKSPACE, "aib_c12_encode_planes: workspace too small");
  if (reinterpret_cast<uintptr_t>(w) & 15) return fail(AIB_EINVAL, "aib_c12_encode_planes: w must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* cnt = static_cast<unsigned long long*>(ws);
  int32_t* rowcnt = reinterpret_cast<int32_t*>(cnt + 256);
  if (cudaMemsetAsync(cnt, 0, 256 * sizeof(unsigned long long), s) != cudaSuccess)
    return launch_check("aib_c12_encode_planes memset");
  const size_t n = static_cast<size_t>(N) * K;
  const int blocks = static_cast<int>(std::min<size_t>((n / 8 + 255) / 256, 4 * static_cast<size_t>(sm_count())));
  codec::hist_kernel<<<std::max(blocks, 1), 256, 0, s>>>(w, n, cnt);
  codec::base_kernel<<<1, 32, 0, s>>>(cnt, base_out);
  codec::planes_kernel<<<N, 128, 0, s>>>(w, N, K, base_out, m8, e4, rowcnt);
  codec::scan_kernel<<<1, 1024, 0, s>>>(rowcnt, N, rp);
  return launch_check("aib_c12_encode_planes");
}

int aib_c12_encode_exceptions(const uint16_t* w, int N, int K, int base, const int32_t* rp, int32_t* er, int32_t* ec,
                              float* ev, void* stream) {
  if (!w || !rp || N <= 0 || K <= 0 || K % codec::CH || base < 0 || base > 241)
    return fail(AIB_EINVAL, "aib_c12_encode_exceptions: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int warps_per_block = 8;
  codec::exc_kernel<<<(N + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(w, N, K, base, rp,
                                                                                                 er, ec, ev);
  return launch_check("aib_c12_encode_exceptions");
}

int aib_c12_decode(const aib_c12* c, int first, int last, void* out, int out_dtype, void* stream) {
  if (!c || !out || !c->m8 || !c->e4 || !c->rp || c->K <= 0 || c->K % codec::CH || c->CH != codec::CH || first < 0 ||
      last > c->N || first >= last || (out_dtype != 0 && out_dtype != 1) || (c->n_exc > 0 && (!c->ec || !c->ev)))
    return fail(AIB_EINVAL, "aib_c12_decode: bad arguments (first=%d last=%d N=%d)", first, last, c ? c->N : -1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (out_dtype)
    return launch(codec::decode_kernel<1>, dim3(last - first), dim3(256), 0, s, "aib_c12_decode", *c, first, last, out);
  return launch(codec::decode_kernel<0>, dim3(last - first), dim3(256), 0, s, "aib_c12_decode", *c, first, last, out);
}

}  // extern "C"
