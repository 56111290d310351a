/*
 * libtk_b200 -- C ABI of the B200 (sm_100a) Transformer layer-stack forward.
 *
 * Plain pointers, 64-bit sizes and a cudaStream_t passed as void*; no torch
 * types. The caller allocates and owns every buffer (device memory on the
 * device that is current for the calling thread); the library keeps only a
 * per-device error word and cached device properties. Every entry point
 * returns TK_OK (0) or a negative tk_status; tk_last_error() then describes
 * the failure (per calling thread). Calls are stream-ordered and do not
 * synchronise, except tk_check_device_errors().
 *
 * Each declaration names the reference interface it replaces
 * (danielfodgaard/transformer-kernel, file:line).
 */
#ifndef TK_B200_H_
#define TK_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tk_status {
  TK_OK = 0,
  TK_ERR_INVALID = -1,      /* bad pointer / size / stride argument            */
  TK_ERR_UNSUPPORTED = -2,  /* valid request outside the kernels' envelope     */
  TK_ERR_LAUNCH = -3,       /* CUDA launch or tensor-map encode failed         */
  TK_ERR_TIMEOUT = -4,      /* a device-side wait gave up (see tk_last_error)  */
  TK_ERR_CUDA = -5,         /* other CUDA runtime error                        */
  TK_ERR_DEVICE = -6        /* kernel reported an error through the error word */
} tk_status;

typedef enum tk_dtype { TK_F32 = 0, TK_F16 = 1 } tk_dtype;

typedef enum tk_epilogue {
  TK_EPI_BIAS = 0,          /* out16 = A W^T + b                                */
  TK_EPI_BIAS_GELU = 1,     /* out16 = gelu_erf(A W^T + b)                      */
  TK_EPI_BIAS_RESID = 2,    /* sum32 = resid + A W^T + b                        */
  TK_EPI_BIAS_RESID_LN = 3  /* sum32 = resid + A W^T + b; out = LN(sum32)       */
} tk_epilogue;

/* Row LayerNorm, optionally fused with a residual add.
 *   y == NULL : out = LN(x)                      -- replaces ln_fwd
 *               (src/fused_kernels.py:164-193); with sum_out non-NULL the
 *               input rows are also copied to sum_out (x's dtype), so a
 *               forward can start its residual stream in its own buffer
 *   y != NULL : s = x + y (fp32 math, stored in x's dtype when sum_out is
 *               non-NULL); out = LN(s)          -- replaces add_ln_fwd
 *               (src/fused_kernels.py:196-238)
 * Statistics in fp32 (mean, centred variance, rsqrt(var + eps)), then the
 * affine, then the cast to out_dtype. x/y/out dtypes: TK_F32 or TK_F16;
 * gamma/beta fp32 [d]. Rows are `ld_*` elements apart. 1 <= d <= 8192.
 * row_len/seq_len: optional prefix-padding lengths (int32 [rows/seq_len]);
 * rows whose position >= row_len[row/seq_len] get s = 0 and out = 0 (the
 * harness's masked_fill of padded tokens, src/torch_transformer_benchmark.py:169-171). */
TK_API int tk_layernorm(const void* x, int x_dtype, int64_t ld_x,
                 const void* y, int y_dtype, int64_t ld_y,
                 void* sum_out, int64_t ld_sum,
                 const float* gamma, const float* beta, float eps,
                 void* out, int out_dtype, int64_t ld_out,
                 const int32_t* row_len, int64_t seq_len,
                 int64_t rows, int64_t d, void* stream);

/* GEMM tile configurations. By default tk_gemm picks the tile by fixed
 * rules (the 256 x 256 CTA-pair tile once there is a wave of them, else the
 * widest single-CTA tile that still gives every SM a tile). A table of
 * measured choices overrides them: tk_gemm_tiles_set records the variant for
 * a GEMM shape (M, N, K, epilogue); later tk_gemm calls with the same
 * (N, K, epilogue) use the entry whose M is nearest on a log scale, when the
 * shape can take that variant (TK_EPI_BIAS_RESID_LN always keeps its
 * one-tile row). Replaces the reference's measured per-shape dispatch table
 * (src/dispatch.py:95-215), which selects settings from sweep results.
 * tk_gemm_tiles_chosen returns the variant tk_gemm would run. */
typedef enum tk_tiles {
  TK_TILES_AUTO = 0,   /* the built-in rules                     */
  TK_TILES_PAIR = 1,   /* 256 x 256 over a CTA pair (N % 256 == 0) */
  TK_TILES_256 = 2,    /* 128 x 256 on one SM (N % 256 == 0)      */
  TK_TILES_128 = 3,    /* 128 x 128 on one SM (N % 128 == 0)      */
  TK_TILES_64 = 4      /* 128 x 64 on one SM                      */
} tk_tiles;
TK_API int tk_gemm_tiles_set(int64_t M, int64_t N, int64_t K, int epilogue, int variant);
TK_API int tk_gemm_tiles_clear(void);
TK_API int tk_gemm_tiles_chosen(int64_t M, int64_t N, int64_t K, int epilogue);

/* out = epilogue(A[M,K] . W[N,K]^T + bias), fp16 operands, fp32 accumulate
 * on the tcgen05 tensor cores. Replaces F.linear (src/optimized.py:572, :627,
 * :632-636) plus the elementwise ops fused into its epilogue (GELU
 * src/optimized.py:635; residual add + LayerNorm src/fused_kernels.py:196-238).
 *   A     : fp16 [M, K], row stride lda (elements), lda % 8 == 0
 *   W     : fp16 [N, K] (nn.Linear.weight as-is), row stride ldw, ldw % 8 == 0
 *   bias  : fp32 [N]
 *   TK_EPI_BIAS / _GELU : out fp16 [M, N], ldo % 8 == 0
 *   TK_EPI_BIAS_RESID   : resid fp32 [M, N] (ld_resid), sum_out fp32 (ld_sum)
 *   TK_EPI_BIAS_RESID_LN: as RESID, plus out = LN(sum) with gamma/beta fp32 [N],
 *                         out_dtype TK_F16 or TK_F32; needs N in {64,128,256}
 *   row_len/seq_len : optional prefix-padding lengths [M/seq_len]; rows whose
 *                     position >= row_len[row/seq_len] are written as zeros
 * N % 32 == 0 and K % 8 == 0. `resid` may alias `sum_out` (in-place). */
TK_API int tk_gemm(const void* A, int64_t lda, const void* W, int64_t ldw,
            const float* bias, int epilogue,
            const float* resid, int64_t ld_resid,
            float* sum_out, int64_t ld_sum,
            const float* gamma, const float* beta, float eps,
            void* out, int out_dtype, int64_t ldo,
            const int32_t* row_len, int64_t seq_len,
            int64_t M, int64_t N, int64_t K, void* stream);

/* GEMM + bias + residual add + LayerNorm for any row width up to 4096:
 *   sum_out = resid + A W^T + bias (fp32, may be in place: sum_out == resid)
 *   out     = LN(sum_out) * gamma + beta (fp16 or fp32, statistics in fp32)
 * Replaces F.linear (src/optimized.py:627, :632-636) followed by add_ln_fwd
 * (src/fused_kernels.py:196-238), which the reference fuses for any
 * d_model <= 8192 with its Triton kernel. N in {64, 128, 256} runs
 * tk_gemm's TK_EPI_BIAS_RESID_LN (one tile holds the row; the workspace is
 * unused). N % 256 == 0 with 512 <= N <= 4096 runs the CTA-pair GEMM, whose
 * epilogue publishes per-row partial statistics of each 128-column slice to
 * `workspace`; the last slice of a row to arrive triggers that row's
 * normalisation. The workspace is tk_gemm_resid_ln_workspace_bytes(M, N)
 * bytes (or more), 256-byte aligned, owned by the caller, and must be zero
 * before its first use; every call that completes leaves it as it found it
 * (after a reported device error, zero it again). A workspace sized for M
 * rows serves any call with at most M rows. Calls that share a workspace
 * must not overlap on the GPU. Other arguments as tk_gemm. */
TK_API int64_t tk_gemm_resid_ln_workspace_bytes(int64_t M, int64_t N);
TK_API int tk_gemm_resid_ln_supported(int64_t M, int64_t N, int64_t K);
TK_API int tk_gemm_resid_ln(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                            const float* resid, int64_t ld_resid, float* sum_out, int64_t ld_sum,
                            const float* gamma, const float* beta, float eps,
                            void* out, int out_dtype, int64_t ldo,
                            const int32_t* row_len, int64_t seq_len,
                            int64_t M, int64_t N, int64_t K,
                            void* workspace, int64_t workspace_bytes, void* stream);

/* tk_gemm_resid_ln without the workspace argument. No counterpart in the
 * reference: it is for callers that cannot allocate device memory -- a
 * plugin whose host framework owns every device allocation, a serving loop
 * that may not call the allocator once it runs, a caller with no memory
 * budget left for a workspace -- and so cannot pass one. The scratch lives
 * in an 8 MiB array inside the library (each GPU that loads the library
 * holds it until the process exits); calls needing more than that
 * (tk_gemm_resid_ln_workspace_bytes(M, N) > 8 MiB, e.g. M > 116,000 rows at
 * N = 1024) return TK_ERR_UNSUPPORTED. Allocates nothing. The first call on
 * a device looks the array's address up on that device (the caller's
 * current one), so make it before any stream capture. Every call on a
 * device shares the one array and clears its per-row counters before its
 * kernel runs: calls that overlap on the GPU race with each other. Other
 * arguments and results as tk_gemm_resid_ln; N in {64, 128, 256} needs no
 * scratch and runs tk_gemm. */
TK_API int tk_gemm_resid_ln_static(const void* A, int64_t lda, const void* W, int64_t ldw, const float* bias,
                                   const float* resid, int64_t ld_resid, float* sum_out, int64_t ld_sum,
                                   const float* gamma, const float* beta, float eps,
                                   void* out, int out_dtype, int64_t ldo,
                                   const int32_t* row_len, int64_t seq_len,
                                   int64_t M, int64_t N, int64_t K, void* stream);

/* Attention forward. Replaces F.scaled_dot_product_attention
 * (src/optimized.py:615-624) and flash_attention (src/kernels.py:250-294),
 * with the same contract as the latter: q, k, v are fp16, logically
 * [B, H, S, hd], with arbitrary strides (elements, shared by the three,
 * multiples of 8) and a contiguous last dimension -- e.g. views into the
 * fused [B, S, 3, H, hd] QKV projection (stride_b = 3*S*H*hd,
 * stride_h = hd, stride_s = 3*H*hd). The output is written directly as
 * [B, S, H*hd] fp16 with row stride ld_out (% 8 == 0).
 *   scale  : multiplies q.k after the product (the harness uses hd**-0.5)
 *   causal : mask keys j > query i
 *   kv_len : optional int32 [B]; keys >= kv_len[b] are masked
 * hd in {8, 16, 32, 64, 128, 256} (8 runs the 16-wide kernel with TMA zero-filling
 * the padding; 128 and 256 run a chunked one-tile-per-CTA kernel). */
TK_API int tk_attn_fwd(const void* q, const void* k, const void* v,
                int64_t stride_b, int64_t stride_h, int64_t stride_s,
                void* out, int64_t ld_out,
                int64_t B, int64_t S, int64_t H, int64_t hd, float scale,
                int causal, const int32_t* kv_len, void* stream);

/* Whole-stack forward for small shapes, one launch: every layer of the
 * stack for one sequence per CTA (d_model = ffn = 128, 2 or 4 heads,
 * S <= 128; the harness's case 1 and the appendix shapes around it).
 * Replaces, for those shapes, the whole per-layer sequence that
 * OptimizedTransformer._run_layers_fused (src/optimized.py:488-554) runs
 * kernel by kernel. Inputs:
 *   x, out       : fp32 [B, S, 128], contiguous
 *   w_packed     : fp16 [L * 768, 128] -- per layer the rows of Wq, Wk, Wv
 *                  (384), Wo, W_ffn_in, W_ffn_out (128 each), nn.Linear
 *                  layout [out, in]
 *   vec_packed   : fp32 [L, 1280] -- per layer bq|bk|bv (384), bo, b_in,
 *                  b_out, norm1 weight, norm1 bias, norm2 weight, norm2 bias
 *   final_gamma/beta : fp32 [128]; eps: every LayerNorm's epsilon
 *   row_len      : optional int32 [B] prefix lengths (key padding; padded
 *                  rows are zero in the output)
 *   scale        : attention scale (head_dim**-0.5)
 * Same numerics as the layer-by-layer path (fp16 operands, fp32
 * accumulation, residual stream and statistics). */
TK_API int tk_stack_small_supported(int64_t d, int64_t heads, int64_t ffn, int64_t seq_len);
TK_API int tk_stack_small(const float* x, float* out, const void* w_packed, const float* vec_packed,
                          const float* final_gamma, const float* final_beta, float eps,
                          const int32_t* row_len, int64_t B, int64_t S, int64_t d, int64_t heads,
                          int64_t ffn, int64_t L, int causal, float scale, void* stream);

/* Peer memory and row copies for the batch-split forward over the GPUs of
 * one node, one process per GPU. Replaces the exchange the reference runs
 * serially, batch chunk after batch chunk on one device
 * (src/run_case14.py:153-158 chunked, :279-322 its streamed loop): here the
 * chunks are the ranks' shards, the first rank's buffers hold the whole
 * batch, and every other rank maps them.
 *   tk_peer_export : `handle` (64 bytes, opaque) names the device allocation
 *                    that contains `ptr`; *offset is ptr's byte offset in it.
 *                    Send both to the other processes.
 *   tk_peer_import : maps that allocation into this process (peer access to
 *                    its device is enabled on first touch); *ptr = the
 *                    exported pointer's address here. Importing the same
 *                    allocation again returns the same mapping (counted).
 *   tk_peer_release: drops one import of the mapping that holds `ptr`.
 *   tk_copy_rows   : `rows` rows of `row_bytes` bytes from src (rows
 *                    src_ld bytes apart) to dst (dst_ld bytes apart), stream
 *                    ordered; either side may be an imported peer pointer,
 *                    in which case the copy engines move it over NVLink
 *                    without using any SM. */
TK_API int tk_peer_export(const void* ptr, void* handle, int64_t* offset);
TK_API int tk_peer_import(const void* handle, int64_t offset, void** ptr);
TK_API int tk_peer_release(void* ptr);
TK_API int tk_copy_rows(void* dst, int64_t dst_ld, const void* src, int64_t src_ld, int64_t row_bytes, int64_t rows,
                        void* stream);

/* Guard probes, same meaning as the reference's can_fuse
 * (src/fused_kernels.py:62-64) and attention_supported
 * (src/kernels.py:96-103): 1 when the kernels accept the shape. */
TK_API int tk_layernorm_supported(int64_t d);
TK_API int tk_attn_supported(int64_t head_dim);

/* Synchronise `stream`, then read and clear the current device's error word
 * (set by kernels whose bounded waits gave up). TK_OK or TK_ERR_TIMEOUT /
 * TK_ERR_DEVICE with a message in tk_last_error(). */
TK_API int tk_check_device_errors(void* stream);

/* Limit, in nanoseconds, of every device-side wait in later launches
 * (default 2e9). Returns the previous value. */
TK_API uint64_t tk_set_wait_limit_ns(uint64_t ns);

/* Launch later launch-bound (small) kernels with programmatic stream
 * serialization (1, the default) or plainly (0); returns the previous
 * setting. With it, such a kernel may be scheduled while the previous kernel
 * on the stream drains, and waits on the device (griddepcontrol.wait) for
 * that kernel's results before touching global memory. Large kernels always
 * launch plainly. No counterpart in the reference (its kernels are launched
 * by Triton / PyTorch); results are identical either way. */
TK_API int tk_set_programmatic_launch(int enable);

/* Test hook for failure detection: launches one CTA that waits on an
 * mbarrier nothing arrives on, with the configured limit, so the wait gives
 * up and records TK_ERR_TIMEOUT in the error word. Never faults. */
TK_API int tk_selftest_wait_timeout(void* stream);

/* Message of the last failed call on this thread ("" if none). */
TK_API const char* tk_last_error(void);

/* Library version string. */
TK_API const char* tk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TK_B200_H_ */
