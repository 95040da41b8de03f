/*
 * b200fo.h -- C ABI of libb200fo.so, the B200 (sm_100a) fused dense-operator library.
 *
 * The library replaces the device half of leon062112/icpp-tuning's operator family
 * (kernel/tilelang/gemm/*.py, kernel/tilelang/conv/conv2d*.py).  In the reference the
 * boundary between Python and the GPU is the callable returned by tilelang.compile(...)
 * (kernel/tilelang/gemm/gemm.py:89, gemm_bias_act.py:96, gemm_bias_layernorm.py:164 and
 * :176-181, conv/conv2d.py:290, conv/conv2d_relu.py:155).  Those callables take device
 * tensors, launch one compiled kernel on the current stream and either return a new
 * output tensor (out_idx=[-1]) or write into a caller-provided one (conv).
 *
 * Here every entry point takes plain device pointers, sizes and a cudaStream_t passed as
 * void*.  The caller owns every buffer.  Nothing is synchronised implicitly.  Every
 * function returns FO_OK (0) or a negative FO_E* code; fo_last_error() returns the
 * message of the last failure on the calling host thread.
 */
#ifndef B200FO_H_
#define B200FO_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FO_ABI_VERSION 2

/* ---- return codes ---------------------------------------------------------------- */
#define FO_OK 0
#define FO_EINVAL (-1)      /* bad argument: shape, stride, alignment, dtype, config   */
#define FO_ECUDA (-2)       /* a CUDA runtime / driver call failed                      */
#define FO_EUNSUPPORTED (-3)/* legal request this build does not implement              */
#define FO_ENODEVICE (-4)   /* no sm_100 device current                                */
#define FO_ETIMEOUT (-5)    /* a bounded device-side wait ran out (see fo_device_status)*/

/* ---- element types ---------------------------------------------------------------- */
#define FO_DT_F16 0
#define FO_DT_BF16 1
#define FO_DT_F32 2

/* ---- layout of the B operand (weights) --------------------------------------------- */
#define FO_B_KN 0 /* B[K,N] row-major: N contiguous (reference layout, gemm.py:64)      */
#define FO_B_NK 1 /* B stored as [N,K]: K contiguous ("column-major B", nn.Linear)    */

/* ---- fused epilogues -------------------------------------------------------------- */
#define FO_EPI_NONE 0           /* C = A.B                          (gemm.py:20-21)        */
#define FO_EPI_BIAS 1           /* C = A.B + bias                   (gemm_bias_layernorm.py:86-87) */
#define FO_EPI_BIAS_RELU 2      /* C = relu(A.B + bias)             (gemm_bias_act.py:81-82) */
#define FO_EPI_BIAS_GELU_TANH 3 /* C = gelu_tanh(A.B + bias)        (end2end.py:37-38)     */
#define FO_EPI_BIAS_GELU_ERF 4  /* C = gelu_erf(A.B + bias)         (end2end.py:83)        */
#define FO_EPI_BIAS_LN 5        /* C = LN_N(A.B + bias)*gamma+beta  (gemm_bias_layernorm.py:93-164) */
#define FO_EPI_RELU 6           /* C = relu(A.B), no bias           (conv2d_relu.py:133-139) */
#define FO_EPI_BIAS_RESIDUAL_LN 7 /* C = LN_N(A.B + bias + residual)*gamma+beta, A.B + bias rounded to
                                     the output dtype first       (end2end.py:76-79, :84-87) */
/* conv2d only, BatchNorm in inference form with per-channel vectors of vec_dtype:
 * bn(y) = (y - mean) * rsqrt(var + bn_eps) * gamma + beta */
#define FO_EPI_BN 8          /* Y = bn(conv)                     (conv2d_bn.py:29-45)        */
#define FO_EPI_BN_RELU 9     /* Y = relu(bn(conv))               (conv2d_bn_relu.py:123-137) */
#define FO_EPI_BN_ADD_RELU 10 /* Y = relu(bn(conv) + residual), var clamped at 0
                                                                 (conv_bn_add_relu.py:29-46) */

/* Tile configuration chosen by the autotuner (icpp_tuning_b200.autotuner).  The
 * reference's TuneConfig is (block_M, block_N, block_K, num_stages, num_warps)
 * (kernel/autotuner/cost_model.py:154-178); on sm_100a block_M is the tcgen05 M (128),
 * block_K is one 128-byte swizzle row (64 16-bit elements) and the warp count is fixed
 * by the warp-specialised design, so the free parameters are block_n, stages, group_m
 * and the grid size. */
typedef struct FoTileCfg {
  int32_t block_m;  /* 128 (one CTA) or 256 (a CTA pair, tcgen05 cta_group::2)         */
  int32_t block_n;  /* 64, 128 or 256                                                   */
  int32_t block_k;  /* 64, or 128: two 64-wide K slices per pipeline stage (one barrier  */
                    /* wait and one commit per 8 MMAs instead of 4)                       */
  int32_t stages;   /* shared-memory pipeline depth, 2..8 (bounded by 227 KB)          */
  int32_t group_m;  /* tile raster: 0 = row-major, g>0 = groups of g row blocks        */
  int32_t max_ctas; /* persistent grid size cap; 0 = one CTA per SM                     */
  int32_t swap_ab;  /* conv2d only: 1 = compute Y^T = W^T X^T (M = 128 output channels,  */
                    /* N = block_n output pixels) so few-channel convs use wide MMAs     */
  int32_t split_k;  /* K split of the tiles that do not fill a whole wave of CTAs:        */
                    /* 0 = automatic (by a cost model when under half a wave),            */
                    /* 1 = never, s = 2..16 = s parts                                     */
  int32_t split_mode; /* how split parts are reduced:                                     */
                    /* 0 = automatic (cluster when eligible, else workspace),             */
                    /* 1 = workspace: fp32 partials in the caller's zero-filled workspace */
                    /*     (fo_gemm_workspace_size), the last-arriving part reduces,      */
                    /* 2 = cluster: the s parts of a tile run as one thread-block cluster */
                    /*     and reduce-scatter their partials through distributed shared   */
                    /*     memory, no workspace (gemm with block_m 128, s <= 8, one wave, */
                    /*     not with FO_EPI_BIAS_LN)                                       */
  int32_t ln_mode;  /* FO_EPI_BIAS_LN only: 0 = automatic (one kernel when eligible and  */
                    /*     M x N >= 2^24, where it measured faster),                      */
                    /* 1 = two kernels: the GEMM stores biased rows + slice statistics,   */
                    /*     a row pass normalises them in place,                           */
                    /* 2 = one kernel: each epilogue warp normalises its own stored slice */
                    /*     once every slice of its rows has published its statistics     */
                    /*     (block_n >= 128; a cooperative launch, all CTAs resident)     */
                    /* 3 = one kernel, slices held: each epilogue warp keeps its slice in */
                    /*     the TMEM accumulator until its rows' statistics are merged,    */
                    /*     then normalises and stores it once (block_n >= 128, every row  */
                    /*     block's tiles within fewer raster units than one wave: group_m */
                    /*     0 and tiles_n <= CTAs (pairs); cooperative launch)            */
} FoTileCfg;

/* One GEMM-family call.  A[M,K] row-major (row stride lda elements).  B per b_layout
 * with row stride ldb.  out[M,N] row-major with row stride ldo.  bias/gamma/beta are
 * length-N vectors of type vec_dtype (may be NULL when the epilogue does not read them).
 * For FO_EPI_BIAS_LN the caller provides workspace (fo_gemm_workspace_size bytes,
 * zero-filled before its first use; every call leaves it zeroed) for the per-row slice
 * statistics and the arrival counters of the one-kernel path (FoTileCfg.ln_mode).  After
 * a call that reported FO_ETIMEOUT (fo_device_status) the counters may be left non-zero:
 * zero the workspace again before reusing it. */
typedef struct FoGemmDesc {
  int64_t M, N, K;
  const void* a;
  const void* b;
  const void* bias;
  const void* gamma;
  const void* beta;
  void* out;
  int64_t lda, ldb, ldo;
  int32_t in_dtype;  /* FO_DT_F16 or FO_DT_BF16 (A and B share it)                     */
  int32_t vec_dtype; /* dtype of bias/gamma/beta                                       */
  int32_t out_dtype; /* FO_DT_F16, FO_DT_BF16 or FO_DT_F32                             */
  int32_t b_layout;  /* FO_B_KN or FO_B_NK                                             */
  int32_t epilogue;  /* FO_EPI_*                                                        */
  float eps;         /* LayerNorm epsilon (reference default 1e-5)                      */
  void* workspace;
  size_t workspace_bytes;
  const void* residual; /* FO_EPI_BIAS_RESIDUAL_LN: [M, N] of out_dtype, row stride ldr */
  int64_t ldr;
} FoGemmDesc;

/* NHWC conv2d as implicit GEMM (reference kernel/tilelang/conv/conv2d.py:208-279):
 * x[n,h,w,c], w[kh,kw,c,f] (the reference's weight layout, conv2d.py:224), out[n,oh,ow,f].
 * GEMM view: M = n*oh*ow, N = f, K = kh*kw*c.  Epilogues: NONE, BIAS, RELU, BIAS_RELU,
 * BN, BN_RELU, BN_ADD_RELU (BatchNorm vectors bn_* of vec_dtype; the residual of
 * BN_ADD_RELU is an [n, oh, ow, f] tensor of the 16-bit output dtype). */
typedef struct FoConvDesc {
  int32_t n, h, w, c, f, kh, kw, stride, pad, dil;
  const void* x;
  const void* wgt;
  const void* bias;
  void* out;
  int32_t in_dtype;
  int32_t vec_dtype;
  int32_t out_dtype;
  int32_t epilogue;
  void* workspace;        /* optional, zero-filled: fp32 partials of the split-K tail */
  size_t workspace_bytes; /* (fo_conv2d_workspace_size); NULL / 0 = no split          */
  const void* bn_gamma;   /* BatchNorm epilogues: [f] vectors of vec_dtype            */
  const void* bn_beta;
  const void* bn_mean;
  const void* bn_var;
  float bn_eps;           /* reference defaults: 1e-3 (BN), 1e-5 (BN_RELU, BN_ADD_RELU) */
  const void* residual;   /* BN_ADD_RELU: [n, oh, ow, f] of out_dtype                  */
} FoConvDesc;

/* Replaces: the callable from tilelang.compile(...) for gemm / gemm_bias_act /
 * gemm_bias_layernorm (kernel/tilelang/gemm/gemm.py:84-89, gemm_bias_act.py:91-96,
 * gemm_bias_layernorm.py:167-188).  Launches one persistent kernel on `stream`. */
int fo_gemm(const FoGemmDesc* desc, const FoTileCfg* cfg, void* stream);

/* Bytes of workspace fo_gemm uses for this (desc, cfg).  FO_EPI_BIAS_LN: required (per-row
 * slice statistics and arrival counters, zero-filled once).  Other epilogues: optional room for fp32 partials of a
 * split-K tail -- the tiles of a last, less than half-full wave (or of a problem with
 * fewer tiles than SMs) split along K over idle SMs; it must be zero-filled before its
 * first use and is left zeroed.  Without it (or with 0 returned) tiles are never split. */
size_t fo_gemm_workspace_size(const FoGemmDesc* desc, const FoTileCfg* cfg);

/* Replaces: build_conv2d_kernel(...)(X, W, Y) (kernel/tilelang/conv/conv2d.py:282-290,
 * conv2d_relu.py:146-155).  Writes into desc->out. */
int fo_conv2d(const FoConvDesc* desc, const FoTileCfg* cfg, void* stream);

/* Bytes of optional workspace fo_conv2d uses to split the tiles of a partial last wave
 * along K (zero-filled before first use, left zeroed); 0 when no split applies. */
size_t fo_conv2d_workspace_size(const FoConvDesc* desc, const FoTileCfg* cfg);

/* Legality of a tile config for an op (0 = gemm family, 1 = conv2d) and output dtype:
 * shared memory <= 227 KB, TMEM columns <= 512, tcgen05 shape rules.  Returns FO_OK or
 * FO_EINVAL with the reason in `why`.  Host-only; needs no GPU.  Used by the autotuner's
 * pruning (reference kernel/autotuner/search_space.py:239-286). */
int fo_query_config_legal(int32_t op, int32_t out_dtype, const FoTileCfg* cfg, char* why,
                          size_t why_len);

/* Dynamic shared memory the kernel for (op, cfg) requests, or 0 if illegal. Host-only. */
size_t fo_config_smem_bytes(int32_t op, int32_t out_dtype, const FoTileCfg* cfg);

/* Device status word written by bounded waits that ran out: returns the first error code
 * recorded on `device` since the last clear (0 if none), optionally clearing it.  Reading
 * synchronises the device. */
int fo_device_status(int32_t device, int32_t clear, int32_t* where);

/* Limit, in nanoseconds, of every bounded device-side wait in later launches (default
 * 2e9).  Kernels that exceed it record FO_ETIMEOUT in the device status and return. */
int fo_set_wait_timeout_ns(uint64_t ns);

/* Launches a one-warp kernel whose wait on an mbarrier nothing ever arrives on must run
 * out after timeout_ns; the kernel records FO_ETIMEOUT and returns.  Used by tests of the
 * failure path; it faults nothing.  Synchronises the stream. */
int fo_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/* Message of the last failure on this host thread (copied into buf); returns its code. */
int fo_last_error(char* buf, size_t len);

/* Scratch held by fo_gemm_bias_layernorm_noalloc on every GPU that loads the library. */
#define FO_NOALLOC_LN_SCRATCH_BYTES (8u << 20)

/* No counterpart in the reference.  fo_gemm with FO_EPI_BIAS_LN for callers that cannot
 * allocate device memory -- e.g. a serving process that reserves its whole memory budget
 * at start-up, or a plugin interface that passes inputs and outputs but no allocator.
 * Same arguments and result as fo_gemm (desc->workspace is ignored); the LayerNorm
 * statistics live in a static __device__ array of FO_NOALLOC_LN_SCRATCH_BYTES per GPU
 * instead, and nothing is allocated: no cudaMalloc, no cudaFree.  Problems needing more
 * scratch (fo_gemm_workspace_size > FO_NOALLOC_LN_SCRATCH_BYTES) fail with FO_EINVAL.
 * The first call on a device looks up the array's address (legal under a stream
 * capture too).  Each call clears the array's counters on `stream` (cudaMemsetAsync)
 * and then runs fo_gemm on it, so config checks, the wait limit, fo_device_status and
 * fo_launch_count behave as for fo_gemm.  All calls share the array: calls that overlap
 * on the GPU race and must be serialised. */
int fo_gemm_bias_layernorm_noalloc(const FoGemmDesc* desc, const FoTileCfg* cfg, void* stream);

/* Library version string, e.g. "b200fo 0.2.0 sm_100a abi 2". */
const char* fo_version(void);

/* Number of kernel launches this library has issued from this process. */
uint64_t fo_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* B200FO_H_ */
