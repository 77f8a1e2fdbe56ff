/* ai_b200 -- C ABI of the B200-native (sm_100a) 12-bit-codec decode path.
 *
 * Every entry point replaces one Python launcher or kernel launch of the reference engine
 * (karabilo214/AI, `ramvi/engine/ramvi_engine/...`; cited per function). The reference has no native FFI for
 * this path -- its kernels are Triton launched from Python -- so this header is the boundary a binding
 * (for example through Python ctypes) calls instead of those launchers.
 *
 * Conventions (same contract as the reference launchers, made explicit for C):
 *  - All device pointers are caller-owned; kernels write their outputs in place.
 *  - Calls are stream-ordered on `stream` (a cudaStream_t passed as void*), never allocate device memory
 *    and never synchronise, so they can be captured in CUDA graphs. Scratch memory, where a kernel needs
 *    it, is a caller-provided workspace (`ws`, `ws_bytes`; size from the matching *_workspace query; it must
 *    be zero-filled once before first use -- the kernels leave their counters at zero again).
 *  - Return value: AIB_OK (0) or a negative AIB_E* code; aib_last_error() gives a message for the calling
 *    thread. Shape errors map to the reference's ValueError (e.g. wcomp.py:122-123).
 *  - Device-side failures (a bounded wait that ran out, an out-of-range index in data) never trap: they set
 *    a device status word readable with aib_status_read().
 */
#ifndef AI_B200_H
#define AI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AIB_ABI_VERSION 1

#define AIB_OK 0
#define AIB_EINVAL (-1)     /* bad argument / shape (reference: ValueError)           */
#define AIB_ECUDA (-2)      /* CUDA runtime error at launch                            */
#define AIB_EWORKSPACE (-3) /* workspace missing or too small                          */
#define AIB_ENOTSUP (-4)    /* configuration not supported by this build               */
#define AIB_ESPACE (-5)     /* output capacity too small (two-pass APIs report need)   */

/* device status codes (aib_status_read) */
#define AIB_DEV_TIMEOUT_FULL 101  /* GEMV consumer waited too long for a TMA stage          */
#define AIB_DEV_TIMEOUT_EMPTY 102 /* GEMV producer waited too long for a free stage         */
#define AIB_DEV_BAD_TOKEN 103     /* embedding id outside the vocabulary                     */
#define AIB_DEV_BAD_POS 104       /* KV position outside [0, maxt)                            */
#define AIB_DEV_SAMPLER_CAP 105   /* sampler candidate buffer overflow                        */
#define AIB_DEV_OVERFLOW 106      /* an output list is shorter than its CSR row pointers say  */

/* One 12-bit-encoded matrix W [N, K] (K % CH == 0, CH == 256), device pointers. Same planes as the
 * reference `compress` dict (wcomp.py:13-32): m8 [N,K] = sign<<7|mantissa, e4 [N,K/2] exponent codes
 * (byte i of each 256-chunk holds element i in the low nibble and 128+i in the high nibble), base,
 * CSR exceptions rp [N+1], er/ec [n_exc] (row-major order), ev [n_exc] fp32 values. */
typedef struct aib_c12 {
  const uint8_t* m8;
  const uint8_t* e4;
  const int32_t* rp;
  const int32_t* er;
  const int32_t* ec;
  const float* ev;
  int32_t base;
  int32_t N;
  int32_t K;
  int32_t CH;
  int64_t n_exc;
} aib_c12;

/* ------------------------------------------------------------------------------------ library ---- */
int aib_abi_version(void);
const char* aib_last_error(void);
/* Programmatic dependent launch between consecutive kernels (default on). */
void aib_set_pdl(int enabled);
/* Device status word of the current device: copies it to *out (synchronous) and, if clear != 0, resets it. */
int aib_status_read(int* out, int clear);
/* Test knobs of the current device (synchronous; no reference counterpart), so that tests can make a bounded wait
 * run out without any fault: knob 1 = spin limit of every bounded wait (polls; 0 restores the default, 2^22 polls,
 * far longer than any legitimate wait), knob 2 = 1 makes the wide T = 1 GEMV's producer withhold its copies (its stages
 * never fill, its consumers give up after the spin limit and record AIB_DEV_TIMEOUT_FULL), knob 3 = how many
 * thread-block cluster sizes (16, then 8 CTAs) the decode attention tries for its cluster merge before the
 * ticket merge (default 0: ticket merge only; its feasibility query is not allowed inside a graph capture),
 * knob 4 = the T = 1 GEMV kernel: 3 (default) the tensor-core wide-stage kernel, two CTAs per SM where the
 * shape fits, else one; 4 its one-CTA-per-SM geometry only; 1 the CUDA-core 12 KB-stage kernel (the path for
 * shapes the tensor-core kernel cannot take). Not for production. */
int aib_debug_knob(int knob, int value);

/* ---------------------------------------------------------------------------------- 12-bit codec ---- */
/* Host encoder, bit-exact with `compress` (wcomp.py:13-32). w: bf16 bits [N,K]. Writes m8, e4, rp, *base,
 * *n_exc; writes er/ec/ev when exc_cap >= *n_exc, else returns AIB_ESPACE (call again with room). */
int aib_c12_encode_host(const uint16_t* w, int N, int K, uint8_t* m8, uint8_t* e4, int32_t* rp, int32_t* base,
                        int64_t* n_exc, int32_t* er, int32_t* ec, float* ev, int64_t exc_cap);
/* Device encoder, pass 1 (replaces `compress` run on the GPU at load, core/engine.py:223-224): histogram,
 * base selection, m8/e4 planes and rp. base_out / rp are device pointers; rp[N] is the exception count.
 * ws >= aib_c12_encode_workspace(N) bytes (no zero-fill needed). */
size_t aib_c12_encode_workspace(int N);
int aib_c12_encode_planes(const uint16_t* w, int N, int K, uint8_t* m8, uint8_t* e4, int32_t* rp, int32_t* base_out,
                          void* ws, size_t ws_bytes, void* stream);
/* Device encoder, pass 2: exception lists (row-major) given rp from pass 1. */
int aib_c12_encode_exceptions(const uint16_t* w, int N, int K, int base, const int32_t* rp, int32_t* er,
                              int32_t* ec, float* ev, void* stream);
/* Exact decode of rows [first,last) (replaces `decompress` wcomp.py:35-45 and `decode_rows`
 * prefill_kernels.py:221-231). out_dtype 0: fp32 [last-first, K]; 1: bf16 bits. */
int aib_c12_decode(const aib_c12* c, int first, int last, void* out, int out_dtype, void* stream);

/* --------------------------------------------------------------------------------- codec GEMV ---- */
/* Y[t] (+)= W * xin(X[t]) for t < T (replaces `gemvc1` wcomp.py:118-126 for T == 1 and `gemvc_tc`
 * wcomp.py:233-242 for 1 < T <= 16). mode 0: Y = Wx; 1: Y += Wx; 2: input silu(x[:K]) * x[K:2K], Y += Wx;
 * 3 (gated output, no reference counterpart): W's rows come in (gate_i, up_i) pairs -- rows 2i and 2i+1 --
 *   and Y[i] = silu((Wx)[2i]) * (Wx)[2i+1] for i < N/2 (N even), the MLP's SiLU gate fused into the
 *   gate/up GEMV; T == 1 needs K a multiple of 1024.
 * lnw (bf16 bits [K], may be NULL): RMSNorm prologue of gemvc1_k (wcomp.py:75-86), T == 1 only.
 * x_stride / y_stride: elements between rows of X / Y (ignored for T == 1).
 * ws (optional, T == 1): aib_gemv_c12_workspace(c, 1) bytes, 16-byte aligned and zero-filled once before the
 * first call (it is left zeroed after every call). With it, when that shortens the longest CTA's share, the
 * matrix's (row tile, column group) stages are split evenly over the CTAs and a row tile shared by
 * neighbouring CTAs is completed by the one holding its first stage, adding the parts in a fixed order
 * (deterministic); without it every CTA takes whole row tiles. The workspace is touched only after the
 * previous kernel on the stream has completed, so calls in one stream may share one; calls that may overlap
 * on the GPU (other streams) need separate workspaces. */
size_t aib_gemv_c12_workspace(const aib_c12* c, int T);
int aib_gemv_c12(const aib_c12* c, const float* x, float* y, int T, int x_stride, int y_stride, int mode,
                 const uint16_t* lnw, float eps, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------- prefill GEMM ---- */
/* Y[m] (+)= W * xin(X[m]) for all M prompt rows at once on the tcgen05 tensor cores, W decoded on the fly
 * (replaces prefill.matrix, kernels/prefill.py:66-78, with mm_k, prefill_kernels.py:8-27, and the fp32 weight
 * blocks of dequant_k + exceptions_k, prefill_kernels.py:59-110). X fp32 [M, ldx]; Y fp32 [M, ldy].
 * xmode 0: xin = X[:, :K]; 2: xin = silu(X[:, :K]) * X[:, K:2K]. lnw (bf16 [K] or NULL): RMSNorm of the rows
 * first, as the gemvc1 prologue. ymode 0: Y = ...; 1: Y += ...; 3: W's rows come in (gate, up) pairs and
 * Y[m, i] = silu(row 2i) * row 2i+1 (N even). precision 1: products of bf16(xin) and the exact bf16 weights;
 * 3: xin split into three bf16 parts (products exact in fp32, fp32 accumulation -- the accuracy of the
 * reference's fp32 mm_k). ws: aib_gemm_c12_workspace(M, K, precision) bytes, 16-byte aligned (no zero-fill). */
size_t aib_gemm_c12_workspace(int M, int K, int precision);
int aib_gemm_c12(const aib_c12* W, const float* X, int M, int ldx, int xmode, const uint16_t* lnw, float eps, float* Y,
                 int ldy, int ymode, int precision, void* ws, size_t ws_bytes, void* stream);

/* --------------------------------------------------------------------------- int8 vocab head ---- */
/* Quantised copy of a vocabulary head w (bf16 bits [V, D]) and its error bounds (replaces Head.__init__,
 * generation/head.py:29-50): per row s = float(max|e|/127) (1 if 0), Q = round-half-even(e/s) clamped to
 * +-127 (int8 [V, D]), C1 = max|e - sQ| (1 + 1e-6), C2 = ||e - sQ||_2 (1 + 1e-6), AM = max|e|, all computed in
 * float64 and stored as fp32 [V]. */
int aib_head8_tables(const uint16_t* w, int V, int D, int8_t* Q, float* S, float* C1, float* C2, float* AM,
                     void* stream);
/* Workspace bytes for aib_head8_bounds / aib_head8_greedy (zero-filled once; calls leave it zeroed). */
size_t aib_head8_workspace(int V, int D, int T);
/* Logit bounds for T <= 16 rows of h (fp32 [T, ldh]) (replaces vocab_a_k, kernels/vocab8.py:19-44):
 * HI[t, v] = s_v Q_v.h_t + B (row stride ldhi), B = min(C2 ||h_t||_2, C1 ||h_t||_1) + 2e-4 AM ||h_t||_1,
 * LO[t] = max_v (s_v Q_v.h_t - B). D a multiple of 16, Q 16-byte aligned. */
int aib_head8_bounds(const float* h, int T, int ldh, const int8_t* Q, const float* S, const float* C1,
                     const float* C2, const float* AM, int V, int D, float* HI, int ldhi, float* LO, void* ws,
                     size_t ws_bytes, void* stream);
/* Greedy token per row (replaces Head.pick with temperature 0, generation/head.py:59-88, and vocab_b_k /
 * vocab_c_k, kernels/vocab8.py:46-77): among the rows v with HI[t, v] >= LO[t], the exact fp32 logit of
 * the head row (decoded from the 12-bit codec W [V, D]; each product rounded to fp32, summed in column
 * order, head.py:19-26); out[t] = the argmax, the smallest id on ties. */
int aib_head8_greedy(const float* h, int T, int ldh, const aib_c12* W, const float* HI, int ldhi, const float* LO,
                     int64_t* out, void* ws, size_t ws_bytes, void* stream);
/* Top-k candidates (no reference counterpart; the reference computes exact logits of the whole vocabulary
 * whenever it samples). aib_head8_bounds_topk: as aib_head8_bounds, but LO[t] = the largest over the kernel's
 * warps of each warp's k-th largest s_v Q_v.h_t - B (1 <= k <= 32; k = 1 is aib_head8_bounds), a lower bound
 * of the k-th largest exact logit, so the rows with HI[t, v] >= LO[t] contain every row of the exact top k
 * (ties included). aib_head8_candidate_logits: logits[t, v] (row stride ldl) = the exact logit (as
 * aib_head8_greedy computes it) for those rows and -inf for every other row; a sampler that keeps only the
 * top k then draws exactly what it draws from the full exact logits. */
int aib_head8_bounds_topk(const float* h, int T, int ldh, const int8_t* Q, const float* S, const float* C1,
                          const float* C2, const float* AM, int V, int D, float* HI, int ldhi, float* LO, int k,
                          void* ws, size_t ws_bytes, void* stream);
int aib_head8_candidate_logits(const float* h, int T, int ldh, const aib_c12* W, const float* HI, int ldhi,
                               const float* LO, float* logits, int ldl, void* ws, size_t ws_bytes, void* stream);
/* Exact logits of every vocabulary row for T <= 16 rows of h (fp32 [T, ldh]) from the 12-bit head W [V, D]
 * (replaces the full-vocabulary exact_rows call of Head.pick when sampling, generation/head.py:19-26 and
 * :62-71): out[t, v] (row stride ldo) = sum over d in column order of fp32(w[v,d] * h[t,d]), each product
 * rounded to fp32 and each addition in fp32 -- bit-identical to the reference's Numba loop. */
int aib_head_exact_logits(const float* h, int T, int ldh, const aib_c12* W, float* out, int ldo, void* stream);

/* ------------------------------------------------------------------------------- norm / embed ---- */
/* out[t] = w * x[t] * rsqrt(mean(x[t]^2) + eps)   (replaces rmsg_k, tkernels.py:216-225) */
int aib_rmsnorm(const float* x, const uint16_t* w, float* out, int T, int D, float eps, void* stream);
/* out[t] = fp32(emb[ids[t]])   (replaces Engine._emb, core/engine.py:388-390, done on the device) */
int aib_embed(const uint16_t* emb, const int64_t* ids, int T, int D, int V, float* out, void* stream);
/* Decode-loop bookkeeping (the reference does this on the host, core/engine.py:393-413):
 * next_ids[0] = out_ids[T-1]; *pos += T; if prior != NULL, prior[new_pos % n_prior] = that id (ring of
 * recent ids for the sampler's penalties). Keeps a captured decode step free of host copies. */
int aib_step_advance(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int T, int32_t* prior, int n_prior,
                     void* stream);
/* Batched decode bookkeeping: next_ids[b] = out_ids[b]; pos[b] += 1 for b < B. */
int aib_batch_advance(int64_t* pos, int64_t* next_ids, const int64_t* out_ids, int B, void* stream);

/* -------------------------------------------------------------------------------- attention ---- */
/* T == 1 fused step (replaces rope_attn_k, tkernels.py:164-213): QK-RMSNorm + RoPE of q and k,
 * bf16 round of the current k/v, write to the caches at *pos, GQA attention over 0..pos (flash-decoding
 * split over the context, ordered merge). qkv fp32 [(H+2KV)*HD]; caches bf16 bits [KV, maxt, HD];
 * out fp32 [H*HD]. ws >= aib_attn_workspace(...), zero-filled once. */
size_t aib_attn_workspace(int H, int KV, int HD, int maxt, int T);
int aib_rope_attn_decode(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv,
                         const int64_t* pos, uint16_t* kc, uint16_t* vc, float* out, int H, int KV, int HD,
                         int maxt, float eps, float scale, void* ws, size_t ws_bytes, void* stream);
/* Same step as aib_rope_attn_decode for callers that cannot allocate device memory once running (an
 * embedding application that budgets all device memory itself, or a serving loop that must never enter
 * cudaMalloc). No counterpart in the reference. Its scratch is a fixed 2 MiB array inside the library,
 * held by every GPU that loads it; calls needing more are rejected with AIB_EINVAL. The first call on a
 * device looks the array up (cudaGetSymbolAddress) and should come before any stream capture. All calls
 * share the array: calls that overlap on the GPU race, so serialise them. */
int aib_rope_attn_decode_noalloc(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv,
                                 const int64_t* pos, uint16_t* kc, uint16_t* vc, float* out, int H, int KV, int HD,
                                 int maxt, float eps, float scale, void* stream);
/* Batched decode of B independent sequences (one token each; no reference counterpart -- the reference decodes one
 * sequence, core/engine.py:538-694 -- it is the rope_attn_k step of each): sequence b's qkv row at qkv + b * qkv_ld,
 * its position pos[b], its caches at kc / vc + b * kv_bstride elements, its output row at out + b * out_ld.
 * ws >= aib_attn_batch_workspace(...), zero-filled once. */
size_t aib_attn_batch_workspace(int H, int KV, int HD, int maxt, int B);
int aib_rope_attn_decode_batch(const float* qkv, int qkv_ld, const uint16_t* qn, const uint16_t* kn, const float* inv,
                               const int64_t* pos, uint16_t* kc, uint16_t* vc, long long kv_bstride, float* out,
                               int out_ld, int B, int H, int KV, int HD, int maxt, float eps, float scale, void* ws,
                               size_t ws_bytes, void* stream);
/* Batched prologue (replaces qk_rope_cache_k, tkernels.py:82-120): q of tokens t < T normed+rotated into
 * q [T, H*HD]; k, v rows written at *pos + t. */
int aib_qk_rope_cache(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv, const int64_t* pos,
                      float* q, uint16_t* kc, uint16_t* vc, int T, int H, int KV, int HD, int maxt, float eps,
                      void* stream);
/* Batched causal attention over the cache (replaces attn_k, tkernels.py:123-150, and the prefill att_k,
 * prefill_kernels.py:30-56): token t attends 0..*pos + t. q [T, H*HD] -> out [T, H*HD]. */
int aib_attn_cached(const float* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos, float* out, int T,
                    int H, int KV, int HD, int maxt, float scale, void* ws, size_t ws_bytes, void* stream);
/* Causal attention of a whole prompt (replaces att_k / attention, prefill_kernels.py:30-56): row i of q
 * [n, H*HD] (position start + i, already normed and rotated) attends cache positions 0 .. start + i of its
 * group; out [n, H*HD]. Tensor-core flash attention (q and probabilities as three bf16 parts). H / KV in
 * {1, 2, 4, 8}; HD 64 or 128; start + n <= maxt. */
int aib_attn_prefill(const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int n, int start, int H, int KV,
                     int HD, int maxt, float scale, void* stream);

/* ------------------------------------------------------------------------- tensor parallelism ---- */
/* In-place sum of x (fp32 [n], n <= nmax) over the `world` tensor-parallel ranks of one node (replaces, for the
 * decode step's small blocks, the NCCL all-reduce after o_proj and down_proj; the reference has no tensor
 * parallelism, planning/multigpu.py:48-95 splits layers instead). buf_ptrs / flag_ptrs: host arrays of every
 * rank's symmetric buffer (2 * nmax floats, 16-byte aligned) and flag words (world ints, zero before the first
 * call), mapped into this process; epoch: this rank's device counter (int, zero before the first call). Every
 * rank makes the same calls in the same order. The sum runs in rank order, so every rank gets the same bits. A
 * peer that does not arrive within the bounded wait sets AIB_DEV_TIMEOUT_FULL and leaves x unchanged. */
int aib_allreduce_oneshot(float* x, int n, int nmax, const int64_t* buf_ptrs, const int64_t* flag_ptrs, int rank,
                          int world, int* epoch, void* stream);

/* ---------------------------------------------------------------------------------- sampler ---- */
/* Logits-in sampler (replaces GGUFEngine._pick, core/gengine.py:452-469, with Constraint.apply,
 * generation/constrain.py:146-148, and the sampling half of Head.pick, generation/head.py:59-88).
 * Order: penalties (repetition over the set of prior ids: l<0 ? l*r : l/r; presence/frequency:
 * l -= f*count + p*[count>0]) -> bitmask (bit j of word w = token 32w+j, 1 = allowed) -> temperature
 * (<= 0: greedy, first index among maxima) -> top-k (keep z >= k-th largest; 0 = off) -> top-p over the
 * descending order (keep while the exclusive cumsum < top_p) -> inverse CDF with the row's uniform u[b]
 * (index = #(cdf <= u), numpy Generator.choice semantics). Top-k and penalties have no reference
 * counterpart (the reference rejects them, server/validation.py:78-85).
 * prior: int32 [B, n_prior] (ids outside [0,V) ignored); bitmask: int32 [B, ceil(V/32)] or NULL;
 * u: float64 [B] or NULL (greedy only); out_ids: int64 [B]. */
typedef struct aib_sample_params {
  float temperature;
  int32_t top_k;
  float top_p;
  float repetition_penalty;
  float presence_penalty;
  float frequency_penalty;
} aib_sample_params;
/* Workspace (bytes, 16-byte aligned) for the multi-CTA path: one CTA per vocabulary slice computes the
 * slice's max, float64 softmax partial and 64 largest logits, one CTA per row merges them; rows whose
 * result could depend on a token outside those candidates (top_k > 64, a nucleus the 64 largest logits do
 * not cover) are completed by the single-CTA algorithm inside the merge, so the ids are the same either way.
 * ws == NULL (or too small) runs the single-CTA algorithm directly. */
size_t aib_sample_workspace(int B, int V);
int aib_sample(const float* logits, int B, int V, int ld, const aib_sample_params* params, const int32_t* prior,
               int n_prior, const int32_t* bitmask, const double* u, int64_t* out_ids, void* ws, size_t ws_bytes,
               void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AI_B200_H */
