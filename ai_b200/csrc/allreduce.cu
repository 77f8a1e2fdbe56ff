// One-shot all-reduce of fp32 rows across the tensor-parallel ranks of one node, over peer memory (sm_100a).
//
// Replaces, for the decode step's small exchanges (one [T, D] fp32 block after o_proj and after down_proj, 16 KB
// at T = 1 on Qwen3-8B), the NCCL all-reduce the tensor-parallel engine issues there. The layer split it serves is
// the one the survey gives for the path (qkv / gate-up by rows, o / down by input columns, one sum per sublayer);
// the reference itself has no tensor parallelism (its multi-GPU mode splits layers, planning/multigpu.py:48-95).
//
// Design: every rank owns a symmetric buffer (two slots of nmax floats) and a flag word per peer, all mapped into
// every rank's address space (torch symmetric memory). A call with epoch e (a per-rank counter kept on the device,
// so graph replays advance it):
//   1. copies its x into slot e & 1 of its own buffer;
//   2. publishes e into its flag word on every rank (release, system scope, after a system fence);
//   3. waits until every peer's flag word in its own array reached e (acquire, bounded: after the spin limit's polls it
//      records AIB_DEV_TIMEOUT_FULL and returns without touching x);
//   4. sums slot e & 1 of every rank's buffer in rank order -- the same order on every rank, so all ranks hold
//      identical bits -- into x, reading peers' slots over NVLink with loads that bypass L1.
// Two slots suffice: a rank writes slot e & 1 again only at epoch e + 2, after every peer has published e + 1,
// which each does only after finishing its reads of epoch e. Plain peer loads and stores only (no TMA, no
// multicast). One CTA: the blocks are a few KB, so the call is latency-bound (a launch plus one NVLink round
// trip), well under an NCCL all-reduce's.
#include "common.cuh"

namespace aib {
namespace ar {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 1024;

struct Peers {
  float* buf[kMaxRanks];  // rank p's symmetric buffer (2 * nmax floats)
  int* flag[kMaxRanks];   // rank p's flag words [world]: flag[p][q] = last epoch rank q published to p
};

AIB_DEV void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
AIB_DEV int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) oneshot_kernel(float* x, int n, int nmax, Peers pe, int rank, int world,
                                                           int* epoch) {
  __shared__ int e_sh, ok_sh;
  const int tid = threadIdx.x;
  pdl_wait();
  if (tid == 0) {
    e_sh = *epoch + 1;
    ok_sh = 1;
  }
  __syncthreads();
  const int e = e_sh, slot = e & 1;
  float* mine = pe.buf[rank] + static_cast<size_t>(slot) * nmax;
  for (int i = tid; i < n; i += kThreads) mine[i] = x[i];
  __syncthreads();
  if (tid < world) {
    __threadfence_system();
    st_release_sys(pe.flag[tid] + rank, e);
    bool seen = false;
    for (uint32_t k = 0, lim = spin_limit(); k < lim; ++k) {
      if (ld_acquire_sys(pe.flag[rank] + tid) >= e) {
        seen = true;
        break;
      }
    }
    if (!seen) {
      set_status(AIB_DEV_TIMEOUT_FULL);
      ok_sh = 0;
    }
  }
  __syncthreads();
  if (ok_sh) {
    for (int i = tid; i < n; i += kThreads) {
      float acc = 0.0f;
      for (int p = 0; p < world; ++p) acc += __ldcv(pe.buf[p] + static_cast<size_t>(slot) * nmax + i);
      x[i] = acc;
    }
  }
  if (tid == 0) *epoch = e;
  pdl_trigger();
}

}  // namespace ar
}  // namespace aib

using namespace aib;

extern "C" {

int aib_allreduce_oneshot(float* x, int n, int nmax, const int64_t* buf_ptrs, const int64_t* flag_ptrs, int rank,
                          int world, int* epoch, void* stream) {
  if (!x || !buf_ptrs || !flag_ptrs || !epoch || n <= 0 || n > nmax || world < 1 || world > ar::kMaxRanks ||
      rank < 0 || rank >= world)
    return fail(AIB_EINVAL, "aib_allreduce_oneshot: bad arguments (n=%d nmax=%d rank=%d world=%d)", n, nmax, rank,
                world);
  ar::Peers pe{};
  for (int p = 0; p < world; ++p) {
    if (!buf_ptrs[p] || !flag_ptrs[p] || (buf_ptrs[p] & 15) || (flag_ptrs[p] & 3))
      return fail(AIB_EINVAL, "aib_allreduce_oneshot: peer %d pointers", p);
    pe.buf[p] = reinterpret_cast<float*>(buf_ptrs[p]);
    pe.flag[p] = reinterpret_cast<int*>(flag_ptrs[p]);
  }
  return launch(ar::oneshot_kernel, dim3(1), dim3(ar::kThreads), 0, static_cast<cudaStream_t>(stream),
                "aib_allreduce_oneshot", x, n, nmax, pe, rank, world, epoch);
}

}  // extern "C"
