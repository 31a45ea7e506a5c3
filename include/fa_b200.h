/*
 * fa_b200.h -- C ABI of the B200 (sm_100a) attention / MLP hot path.
 *
 * Library: libfa_b200.so (built by cs348k_fast_attention_grammar_b200/build.py).
 * All entry points are stream-ordered and asynchronous on the caller's
 * stream; none of them allocates device memory, and the caller owns every
 * buffer.  Every function returns an fa_status (0 = success); no C++
 * exception crosses this boundary.  Tensors are bf16 (raw 16-bit words)
 * unless the name says f16 or f32, pointers are device pointers, strides are
 * in elements.
 *
 * Reference interfaces replaced (paths inside nriedman/cs348k-fast-attention-grammar):
 *   fa_attn_fwd  <- the attention operator behind the kernel-module protocol
 *                   that bench.py:14-20 times: the host callable fn(KT, Q, V)
 *                   emitted at grammar/kernel_ast.py:1267-1287 (e.g.
 *                   runs/attn_full/kernels/best_it24.py:78-99), the torch
 *                   modules pytorch-naive.py:23-65 and flash-attn2-sota.py:41-63,
 *                   and the batched attention(q, k, v) of
 *                   old/kernels/old/naive.py:27-56 / old/benchmark.py:17-21.
 *   fa_attn_fwd_f32 <- the same callables at the reference's own fp32 2-D
 *                   problem (fn(KT, Q, V) with fp32 cupy arrays), staging to
 *                   bf16 on the device instead of host-side casts.
 *   fa_mlp_fwd   <- the host callable emitted for the MLP program of
 *                   run_mlp_search.py:42-127 (stages h = X@W1, a = act(h),
 *                   y = a@W2 at :58-69).
 *   fa_gemm_act  <- one matmul stage with its pointwise epilogue, the
 *                   "matmul" reduction rule grammar/kernel_ast.py:207-211
 *                   (ct.mma K-loop) followed by the relu stage of
 *                   run_mlp_search.py:62-64.
 *   *_f16        <- the same operators at the reference harnesses' default
 *                   dtype, fp16 (bench.py:32 DTYPE_MAP, old/benchmark.py:96
 *                   --dtype fp16, old/kernels/old/naive.py:27-56).
 *   fa_attn_fwd_f32_batched <- the fp32 [B, H, S, D] problem of the
 *                   reference's seeded runs (run_attention_search.py:169-181,
 *                   BASELINE cfg0), one call for all (batch, head) pairs.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fa_status {
  FA_OK = 0,
  FA_ERR_NULL = 1,         /* a required pointer is NULL                        */
  FA_ERR_SHAPE = 2,        /* a dimension is <= 0 or too large                  */
  FA_ERR_HEAD_DIM = 3,     /* head dim not supported (attention: 8..128, x8)    */
  FA_ERR_ALIGN = 4,        /* pointer or stride not 16-byte aligned (TMA rule)  */
  FA_ERR_STRIDE = 5,       /* innermost stride is not 1                         */
  FA_ERR_TMA = 6,          /* cuTensorMapEncodeTiled rejected the tensor        */
  FA_ERR_LAUNCH = 7,       /* kernel launch failed (cudaGetLastError)           */
  FA_ERR_DRIVER = 8,       /* driver entry point unavailable                    */
  FA_ERR_DEVICE = 9,       /* current device is not sm_100 (B200 class)         */
  FA_ERR_ARG = 10,         /* an enum argument is out of range                  */
  FA_ERR_TIMEOUT = 11,     /* a kernel wait ran out (read by fa_device_status)  */
  FA_ERR_CUDA = 12,        /* another CUDA runtime call failed                  */
  FA_ERR_SCRATCH = 13      /* problem exceeds fa_mlp_fwd_noalloc's fixed buffer */
} fa_status;

typedef enum fa_f32_precision {
  FA_F32_BF16 = 0,         /* fp32 operands rounded to bf16 (8 significant bits) */
  FA_F32_SPLIT = 1         /* bf16 hi + lo split, three products per GEMM        */
} fa_f32_precision;

typedef enum fa_activation {
  FA_ACT_NONE = 0,
  FA_ACT_RELU = 1,         /* run_mlp_search.py:62-64                           */
  FA_ACT_GELU_TANH = 2     /* 0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3)))           */
} fa_activation;

/* Human-readable text for a status code (static storage). */
const char* fa_strerror(int status);

/* Library version as major*10000 + minor*100 + patch. */
int fa_version(void);

/*
 * Fused attention forward  O = softmax(Q K^T * scale [+ causal mask]) V.
 *   q, k, v, o : [B, H, S, D] bf16, element strides
 *                strides[0..3] = q (b, h, s, d), strides[4..7] = k,
 *                strides[8..11] = v, strides[12..15] = o; every d-stride must
 *                be 1 and every other stride a multiple of 8 elements.
 *   D          : 8 .. 128, a multiple of 8 (D <= 64 runs the four-tile
 *                kernel, larger D the two-tile kernel; the head dim is
 *                zero-padded to the kernel's width on chip, never in memory).
 *   causal     : nonzero = key j visible to query i iff j <= i.
 *   scale      : softmax scale (pass 1/sqrt(D) for the reference's math).
 *   stream     : cudaStream_t (NULL = legacy default stream).
 * Computes in fp32 (tcgen05 bf16 MMAs with fp32 accumulation in TMEM).
 * With more work units (256 query rows at D = 128, 512 at D = 64; fewer
 * rows when the problem would leave most SMs idle, and at D <= 64 without a
 * causal mask a last partial wave of units split into halves) than SMs
 * the kernel runs persistent and takes units from one of 1024 library-owned
 * device counters, handed out round-robin per call and reset by the launch
 * that used it; a counter is shared only if 1024 further calls are issued
 * while a launch that holds it is still queued or running (for instance
 * replays of separately captured CUDA graphs run concurrently).
 */
int fa_attn_fwd(const void* q, const void* k, const void* v, void* o, int B, int H, int S,
                int D, const int64_t* strides, int causal, float scale, void* stream);

/*
 * fa_attn_fwd with fp16 Q, K, V and O (raw 16-bit words): the same kernels
 * with fp16 tensor-core operands (P is rounded to fp16 for O += P V),
 * fp32 accumulation and softmax.  Arguments and rules as fa_attn_fwd.
 */
int fa_attn_fwd_f16(const void* q, const void* k, const void* v, void* o, int B, int H, int S,
                    int D, const int64_t* strides, int causal, float scale, void* stream);

/*
 * The reference's own 2-D fp32 problem in one call (the kernel-module
 * callables fn(KT, Q, V) of pytorch-naive.py:23 and of every emitted module,
 * grammar/kernel_ast.py:1267-1287, and fn(K, Q, V) of flash-attn2-sota.py:41
 * on one (batch, head) pair):
 *   q [N, D], v [N, D], o [N, D] fp32, contiguous;
 *   k [N, D] fp32 (k_transposed = 0) or KT [D, N] fp32 (k_transposed = 1);
 *   ws         : bf16 workspace of 3 * N * D elements (16-byte aligned), where
 *                q, k, v are staged in bf16 (one launch) for the tensor cores;
 *   D          : as for fa_attn_fwd; causal, scale, stream as for fa_attn_fwd.
 * Two launches (staging, attention); O is written in fp32 by the attention
 * epilogue.  Inputs are rounded to bf16, accumulation is fp32.
 */
int fa_attn_fwd_f32(const void* q, const void* k, const void* v, void* o, void* ws, int N,
                    int D, int k_transposed, int causal, float scale, void* stream);

/*
 * fp32 attention for batched tensors: q, v, o contiguous [B, H, S, D] fp32,
 * k contiguous [B, H, S, D] (k_transposed = 0) or [B, H, D, S] (1).  Two
 * launches for all pairs: staging to bf16, then the attention with an fp32
 * epilogue.  precision:
 *   FA_F32_BF16  : operands rounded to bf16 (as fa_attn_fwd_f32);
 *                  ws = 3 * B * H * S * D bf16 elements;
 *   FA_F32_SPLIT : each operand x staged as hi = bf16(x) and lo = bf16(x - hi),
 *                  and S = Qh Kh^T + Qh Kl^T + Ql Kh^T, O = Ph Vh + Ph Vl + Pl Vh
 *                  accumulated in fp32 (about 16 significant bits; three times
 *                  the tensor-core work); D <= 64; ws = 3 * B * H * S * 128.
 * ws is 16-byte aligned.
 */
int fa_attn_fwd_f32_batched(const void* q, const void* k, const void* v, void* o, void* ws,
                            int B, int H, int S, int D, int k_transposed, int causal,
                            float scale, int precision, void* stream);

/*
 * C[M, N] = act(A[M, K] @ B[K, N]) in bf16 with fp32 accumulation.
 *   A row-major with row stride lda (K contiguous); B row-major [K, N] with
 *   row stride ldb (N contiguous); C row-major with row stride ldc.
 *   K and N must be multiples of 64, M any positive value; lda, ldb, ldc
 *   multiples of 8.
 */
int fa_gemm_act(const void* a, const void* b, void* c, int M, int N, int K, int64_t lda,
                int64_t ldb, int64_t ldc, int act, void* stream);

/* fa_gemm_act with fp16 A, B and C (fp32 accumulation).  Same rules. */
int fa_gemm_act_f16(const void* a, const void* b, void* c, int M, int N, int K, int64_t lda,
                    int64_t ldb, int64_t ldc, int act, void* stream);

/*
 * MLP block Y[M, K] = act(X[M, K] @ W1[K, N]) @ W2[N, K]   (all row-major bf16).
 *   hidden : caller-owned [M, N] bf16 workspace that receives act(X @ W1).
 *   K, N multiples of 64.  act = FA_ACT_GELU_TANH for the benchmark block,
 *   FA_ACT_RELU for the reference's.
 */
int fa_mlp_fwd(const void* x, const void* w1, const void* w2, void* hidden, void* y, int M,
               int K, int N, int act, void* stream);

/* fa_mlp_fwd with fp16 X, W1, W2, hidden and Y (fp32 accumulation). */
int fa_mlp_fwd_f16(const void* x, const void* w1, const void* w2, void* hidden, void* y, int M,
                   int K, int N, int act, void* stream);

/*
 * The reference's full MLP block (run_mlp_search.py:42-127, checked by its
 * verify at :138-149):
 *   hidden = relu(X @ W1)            [M, N]  caller-owned bf16 workspace
 *   resid  = hidden @ W2 + X         [M, K]  caller-owned bf16 workspace
 *                                            (residual added in GEMM 2's epilogue)
 *   out    = (resid - mean) / sqrt(var + eps) over each row (no affine)
 * K, N multiples of 64; K <= 8192 (the LayerNorm row stays in registers).
 */
int fa_mlp_ln_fwd(const void* x, const void* w1, const void* w2, void* hidden, void* resid,
                  void* out, int M, int K, int N, float eps, void* stream);

/*
 * Row LayerNorm without affine parameters: out[i, :] = (in[i, :] - mean_i) /
 * sqrt(var_i + eps), population variance, computed in fp32 (the LayerNorm
 * stage of run_mlp_search.py:76-93).  N a multiple of 8, N <= 8192; row
 * strides multiples of 8 elements.
 */
int fa_layernorm_rows(const void* in, void* out, int M, int N, int64_t ld_in, int64_t ld_out,
                      float eps, void* stream);

/*
 * fa_mlp_fwd without any device allocation: the same MLP block, with the
 * hidden activation kept in a fixed array inside the library instead of a
 * caller-provided buffer.  No counterpart in the reference.
 *   For callers that cannot call cudaMalloc or any allocator -- a plugin
 *   running inside a host whose memory pools it does not own, code that
 *   must not allocate while a CUDA graph is being built or while another
 *   component holds the device's memory budget.  They still pass X, W1, W2
 *   and Y.
 *   Limit: M * N <= 8,388,608 hidden elements (a 16 MiB bf16 array that every
 *   GPU loading the library keeps until the process exits); larger problems
 *   return FA_ERR_SCRATCH.  Other shape rules as fa_mlp_fwd.
 *   The first call on each device looks up the array's device address
 *   (cudaGetSymbolAddress); make that first call before any stream capture.
 *   All calls share the one array and it keeps the last call's contents
 *   (every element a call reads it first writes), so calls that may run at
 *   the same time on the GPU -- on different streams, or from different
 *   threads -- race and must be serialised by the caller.
 */
int fa_mlp_fwd_noalloc(const void* x, const void* w1, const void* w2, void* y, int M, int K,
                       int N, int act, void* stream);

/*
 * Failure-detection self test: launches one CTA that waits on an mbarrier no
 * one ever arrives on, with a limit of limit_us microseconds (1 .. 10^6).  The
 * bounded wait gives up, records FA_ERR_TIMEOUT in the device status word and
 * the kernel returns normally (no trap, no fault), so the context stays
 * usable; read the result with fa_device_status().  Every wait inside the
 * library's kernels is bounded the same way (limit 1 s).  Reference analog:
 * the search's compile timeout (grammar/optimization.py:57-62,267-280), which
 * turns a hung compile into a recorded failure.
 */
int fa_selftest_wait_timeout(int limit_us, void* stream);

/*
 * Self test of the attention softmax's exponentials on the device: for the
 * n fp32 values x, writes out[i] = the FMA-pipe 2^x (Cody-Waite style
 * round-to-nearest range reduction, degree-3 minimax polynomial, exponent
 * add), out[n + i] = the same computed two at a time with paired fp32
 * instructions, and out[2n + i] = ex2.approx(x) (MUFU).  out holds 3n
 * floats.  These are the routines the attention kernels call.  Reference
 * analog: the exp stage that run_attention_search.py:64-67 lowers to ct.exp.
 */
int fa_selftest_exp2(const float* x, float* out, int n, void* stream);

/*
 * Reads and clears the device-side status word of the current device
 * (FA_OK, or FA_ERR_TIMEOUT when a kernel's bounded wait ran out).
 * Synchronises the device.
 */
int fa_device_status(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
