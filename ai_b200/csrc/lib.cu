// Single translation unit for libai_b200.so (device symbols such as the status word are shared by all
// kernels without relocatable device code).
#include "runtime.cu"
#include "codec.cu"
#include "gemv.cu"
#include "gemm.cu"
#include "norm.cu"
#include "attn.cu"
#include "attn_noalloc.cu"
#include "pattn.cu"
#include "sampler.cu"
#include "head8.cu"
#include "exact.cu"
#include "allreduce.cu"
