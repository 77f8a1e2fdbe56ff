// RMSNorm rows, embedding gather and decode-loop bookkeeping.
//   aib_rmsnorm: reference rmsg_k (`ramvi/engine/ramvi_engine/kernels/tkernels.py:216-225`)
//   aib_embed:   reference Engine._emb (`core/engine.py:388-390`), done on the device from device ids
#include "common.cuh"

namespace aib {
namespace norm {

__global__ void rms_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w, float* __restrict__ out, int D,
                           float eps) {
  pdl_wait();
  const int t = blockIdx.x;
  const float* xr = x + static_cast<size_t>(t) * D;
  float ss = 0.0f;
  // One summation order whatever the row's alignment: groups of four columns per thread, the tail after.
  // Aligned rows load each group with one 16-byte load; others load the same four values one by one.
  const bool vec = !(reinterpret_cast<uintptr_t>(xr) & 15);
#pragma unroll 4
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
    const float4 v = vec ? reinterpret_cast<const float4*>(xr)[i]
                         : make_float4(xr[4 * i], xr[4 * i + 1], xr[4 * i + 2], xr[4 * i + 3]);
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  for (int i = (D & ~3) + threadIdx.x; i < D; i += blockDim.x) ss += xr[i] * xr[i];
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  float* o = out + static_cast<size_t>(t) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) o[i] = bf16_to_f32(w[i]) * (xr[i] * r);
  pdl_trigger();
}

__global__ void embed_kernel(const uint16_t* __restrict__ emb, const int64_t* __restrict__ ids, int D, int V,
                             float* __restrict__ out) {
  pdl_wait();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) set_status(AIB_DEV_BAD_TOKEN);
    id = 0;
  }
  const uint16_t* row = emb + static_cast<size_t>(id) * D;
  float* o = out + static_cast<size_t>(t) * D;
  if ((D & 7) == 0 && !(reinterpret_cast<uintptr_t>(row) & 15) && !(reinterpret_cast<uintptr_t>(o) & 15)) {
    // 8 values per 16-byte load, all of a thread's loads in flight together (one HBM round trip)
#pragma unroll 4
    for (int i = threadIdx.x; i < D / 8; i += blockDim.x) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(row) + i);
      float4* o4 = reinterpret_cast<float4*>(o) + 2 * i;
      o4[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                          __uint_as_float(v.y & 0xFFFF0000u));
      o4[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u), __uint_as_float(v.w << 16),
                          __uint_as_float(v.w & 0xFFFF0000u));
    }
  } else {
    for (int i = threadIdx.x; i < D; i += blockDim.x) o[i] = bf16_to_f32(row[i]);
  }
  pdl_trigger();
}

// The last sampled id becomes the next step's input and the position advances by the tokens processed.
__global__ void advance_kernel(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int T, int32_t* prior,
                               int n_prior) {
  pdl_wait();
  if (threadIdx.x == 0) {
    const int64_t tok = out_ids[T - 1];
    const int64_t p = *pos + T;
    next_ids[0] = tok;
    if (prior && n_prior > 0 && p >= 0) prior[p % n_prior] = static_cast<int32_t>(tok);
    *pos = p;
  }
  pdl_trigger();
}

// Batched decode: sequence b's sampled id becomes its next input and its position advances by one.
__global__ void batch_advance_kernel(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int B) {
  pdl_wait();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    next_ids[b] = out_ids[b];
    pos[b] += 1;
  }
  pdl_trigger();
}

}  // namespace norm
}  // namespace aib

using namespace aib;

extern "C" {

int aib_rmsnorm(const float* x, const uint16_t* w, float* out, int T, int D, float eps, void* stream) {
  if (!x || !w || !out || T <= 0 || D <= 0) return fail(AIB_EINVAL, "aib_rmsnorm: bad arguments");
  return launch(norm::rms_kernel, dim3(T), dim3(256), 0, static_cast<cudaStream_t>(stream), "aib_rmsnorm", x, w, out,
                D, eps);
}

int aib_embed(const uint16_t* emb, const int64_t* ids, int T, int D, int V, float* out, void* stream) {
  if (!emb || !ids || !out || T <= 0 || D <= 0 || V <= 0) return fail(AIB_EINVAL, "aib_embed: bad arguments");
  return launch(norm::embed_kernel, dim3(T), dim3(256), 0, static_cast<cudaStream_t>(stream), "aib_embed", emb, ids, D,
                V, out);
}

int aib_step_advance(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int T, int32_t* prior, int n_prior,
                     void* stream) {
  if (!pos || !next_ids || !out_ids || T <= 0 || n_prior < 0) return fail(AIB_EINVAL, "aib_step_advance: bad arguments");
  return launch(norm::advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), "aib_step_advance", pos,
                next_ids, out_ids, T, prior, n_prior);
}

int aib_batch_advance(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int B, void* stream) {
  if (!pos || !next_ids || !out_ids || B <= 0) return fail(AIB_EINVAL, "aib_batch_advance: bad arguments");
  return launch(norm::batch_advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                "aib_batch_advance", pos, next_ids, out_ids, B);
}

}  // extern "C"
