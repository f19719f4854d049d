/*
 * neso_b200.h — C ABI of the Neso B200 kernel library (sm_100a).
 *
 * Every kernel that Neso compiles and benchmarks is exported here under the
 * reference kernel's name, with the reference's arguments in the reference's
 * order. The rule that turns a reference launch into a call is uniform:
 *
 *   neso_<kernel>(<runtime args in reference order>,
 *                 <the reference kernel's constexpr parameters, as int32>,
 *                 grid_x, grid_y, grid_z,      // the reference launch grid
 *                 stream)                      // cudaStream_t, NULL = legacy
 *
 * The reference grid is validated against the problem it implies (a mismatch
 * returns NESO_ERR_GRID); the kernels then launch their own B200 grid. The
 * caller owns every buffer; pointers are device pointers. All calls are
 * asynchronous on `stream`, thread-safe and never abort: they return a status
 * code, and neso_last_error_string() gives the thread's last message.
 *
 * Extended entry points (neso_fa2_*, neso_*_mnk, neso_w4a16_*) cover the
 * multi-head, causal, relative-position-table and packed-int4 variants that
 * have no reference kernel; each says so.
 */
#ifndef NESO_B200_H
#define NESO_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NESO_API __attribute__((visibility("default")))
#else
#define NESO_API
#endif

/* A CUDA stream (cudaStream_t / CUstream). NULL selects the legacy stream. */
typedef void* neso_stream_t;

/* Status codes. The reference raises RuntimeError on Metal pipeline/command
 * buffer failures (src/neso/backend/driver.py:138-176, :314-317); these are the
 * C equivalents. */
#define NESO_OK 0
#define NESO_ERR_INVALID_ARG (-1)    /* null pointer, negative size, bad constexpr */
#define NESO_ERR_MISALIGNED (-2)     /* pointer/stride alignment the kernel needs */
#define NESO_ERR_UNSUPPORTED (-3)    /* shape or layout this kernel does not implement */
#define NESO_ERR_GRID (-4)           /* reference grid inconsistent with the problem */
#define NESO_ERR_LAUNCH (-5)         /* CUDA runtime / driver error */
#define NESO_ERR_DEVICE_TIMEOUT (-6) /* a bounded device-side wait expired */
#define NESO_ERR_NO_DEVICE (-7)

/* ------------------------------------------------------------- runtime -- */
NESO_API const char* neso_last_error_string(void);
NESO_API int neso_version(void);
/* Select the CUDA device used by subsequent calls from this thread. */
NESO_API int neso_set_device(int device);
/* Synchronise `device` and read its status word: *code is 0 when no device
 * wait has timed out since the last neso_clear_device_status(). Returns
 * NESO_ERR_DEVICE_TIMEOUT when *code is non-zero. `where`, `block`, `thread`
 * (any may be NULL) locate the first failing wait. */
NESO_API int neso_device_status(int device, int* code, int* where, int* block, int* thread);
NESO_API int neso_clear_device_status(int device);
/* Self-test of the bounded-wait machinery: launches one CTA that waits on an
 * mbarrier nothing arrives at, with a budget of `budget_us` microseconds, and
 * returns the status the kernel reported (NESO_ERR_DEVICE_TIMEOUT expected). */
NESO_API int neso_selftest_wait_timeout(int budget_us, neso_stream_t stream);
/* JSON launch metadata for a kernel name, same keys as the reference's
 * AOTResult.to_metadata() (src/neso/aot_compile.py:108-117). NULL if unknown. */
NESO_API const char* neso_kernel_metadata(const char* kernel_name);

/* ---------------------------------------------------------- elementwise -- */
/* windows/kernels.py:7-15  vector_add(x, y, output, n_elements, BLOCK_SIZE)
 * (== tests/test_aot.py:17-28 add_kernel). Reference grid: (cdiv(n, BLOCK_SIZE), 1, 1).
 * fp32; output[i] = x[i] + y[i] for i < n_elements. */
NESO_API int neso_vector_add(const float* x, const float* y, float* output, int32_t n_elements, int32_t BLOCK_SIZE,
                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_aot.py:17-28 add_kernel(x_ptr, y_ptr, z_ptr, n_elements, BLOCK_SIZE). */
NESO_API int neso_add_kernel(const float* x_ptr, const float* y_ptr, float* z_ptr, int32_t n_elements, int32_t BLOCK_SIZE,
                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* windows/kernels.py:18-22  scale(x, output, factor, n_elements, BLOCK_SIZE).
 * output[i] = x[i] * factor. */
NESO_API int neso_scale(const float* x, float* output, float factor, int32_t n_elements, int32_t BLOCK_SIZE,
               uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);

/* ----------------------------------------- LLM building blocks (rowops) -- */
/* tests/test_advanced12.py:104-120  rmsnorm_kernel(x_ptr, weight_ptr, out_ptr,
 *   row_stride, n_cols, eps, BLOCK_SIZE). Reference grid: (M, 1, 1), one row per
 *   program: out = x / sqrt(sum(x^2) / n_cols + eps) * w over the first
 *   min(BLOCK_SIZE, n_cols) columns of each row. fp32. */
NESO_API int neso_rmsnorm_kernel(const float* x_ptr, const float* weight_ptr, float* out_ptr, int32_t row_stride,
                        int32_t n_cols, float eps, int32_t BLOCK_SIZE, uint32_t grid_x, uint32_t grid_y,
                        uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:135-153  residual_rmsnorm_kernel(x_ptr, residual_ptr,
 *   weight_ptr, out_ptr, row_stride, n_cols, eps, BLOCK_SIZE): RMSNorm of
 *   h = x + residual. Reference grid: (M, 1, 1). */
NESO_API int neso_residual_rmsnorm_kernel(const float* x_ptr, const float* residual_ptr, const float* weight_ptr,
                                 float* out_ptr, int32_t row_stride, int32_t n_cols, float eps, int32_t BLOCK_SIZE,
                                 uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:156-176  rope_kernel(x_ptr, cos_ptr, sin_ptr, out_ptr,
 *   seq_len, head_dim, BLOCK_D). x, out [seq_len, head_dim], cos/sin
 *   [seq_len, head_dim/2]; rotates pairs (d, d + head_dim/2) for
 *   d < min(BLOCK_D, head_dim/2). Reference grid: (seq_len, 1, 1). */
NESO_API int neso_rope_kernel(const float* x_ptr, const float* cos_ptr, const float* sin_ptr, float* out_ptr,
                     int32_t seq_len, int32_t head_dim, int32_t BLOCK_D, uint32_t grid_x, uint32_t grid_y,
                     uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:123-132  silu_kernel(x_ptr, out_ptr, n, BLOCK):
 *   out = x * sigmoid(x). Reference grid: (cdiv(n, BLOCK), 1, 1). */
NESO_API int neso_silu_kernel(const float* x_ptr, float* out_ptr, int32_t n, int32_t BLOCK, uint32_t grid_x,
                     uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_triton_jit.py:55-70  softmax_kernel(output_ptr, input_ptr,
 *   input_row_stride, output_row_stride, n_cols, BLOCK_SIZE): row-wise softmax
 *   over the first min(BLOCK_SIZE, n_cols) columns. Reference grid: (M, 1, 1). */
NESO_API int neso_softmax_kernel(float* output_ptr, const float* input_ptr, int32_t input_row_stride,
                        int32_t output_row_stride, int32_t n_cols, int32_t BLOCK_SIZE, uint32_t grid_x,
                        uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:54-67  per_channel_dequant_kernel(x_int8_ptr,
 *   scale_ptr, zero_ptr, out_ptr, n_rows, n_cols, BLOCK_M, BLOCK_N):
 *   out = (x - zero[col]) * scale[col]; x held as int32 (the reference test
 *   passes int32, :222). Reference grid: (cdiv(n_rows, BLOCK_M), cdiv(n_cols, BLOCK_N), 1). */
NESO_API int neso_per_channel_dequant_kernel(const int32_t* x_int8_ptr, const float* scale_ptr, const float* zero_ptr,
                                    float* out_ptr, int32_t n_rows, int32_t n_cols, int32_t BLOCK_M, int32_t BLOCK_N,
                                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:69-84  grouped_dequant_kernel(x_int8_ptr, scale_ptr,
 *   zero_ptr, out_ptr, n, group_size, BLOCK): out[i] = (x[i] - zero[i / gs]) *
 *   scale[i / gs]; x held as int32. Reference grid: (cdiv(n, BLOCK), 1, 1). */
NESO_API int neso_grouped_dequant_kernel(const int32_t* x_int8_ptr, const float* scale_ptr, const float* zero_ptr,
                                float* out_ptr, int32_t n, int32_t group_size, int32_t BLOCK, uint32_t grid_x,
                                uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* tests/test_advanced12.py:87-101  quantize_kernel(x_ptr, scale_ptr, out_ptr, n,
 *   BLOCK): q = x / scale[0], rounded as q +/- 0.5 truncated toward zero,
 *   clamped to [-128, 127], stored as int32. Reference grid: (cdiv(n, BLOCK), 1, 1). */
NESO_API int neso_quantize_kernel(const float* x_ptr, const float* scale_ptr, int32_t* out_ptr, int32_t n, int32_t BLOCK,
                         uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);

/* ------------------------------------------------------ flash attention -- */
/* tests/test_flash_attention.py:149-152
 *   flash_attention_fwd(Q, K, V, O, N, stride_qo, stride_kv, scale), constexpr d.
 * Single head. Q, K, V fp16 [N, d] with row strides stride_qo / stride_kv
 * (elements), O fp32 [N, d] with row stride stride_qo. HEAD_DIM = d in {64, 128}.
 * Reference grid: (N / BM, 1, 1) with the reference's BM (a power of two in
 * [8, 128]); N must be a multiple of that BM, as in the reference. */
NESO_API int neso_flash_attention_fwd(const void* Q, const void* K, const void* V, float* O, int32_t N, int32_t stride_qo,
                             int32_t stride_kv, float scale, int32_t HEAD_DIM, uint32_t grid_x, uint32_t grid_y,
                             uint32_t grid_z, neso_stream_t stream);

/* tests/test_rel_pos_fa2.py:157-162
 *   rel_pos_fa2_fwd(Q, K, V, bias, O, T, stride, scale, stride_h, bias_stride_h).
 * Multi-head; Q, K, V, bias and O are fp16. Q/K/V/O are [nh, T, d] (row stride
 * `stride`, head stride `stride_h`), bias is a dense [nh, T, T] table (head
 * stride bias_stride_h, row stride T); scores = (Q K^T + bias) * scale
 * (tests/test_rel_pos_fa2.py:202-206). Reference grid: (T / BM, nh, 1). */
NESO_API int neso_rel_pos_fa2_fwd(const void* Q, const void* K, const void* V, const void* bias, void* O, int32_t T,
                         int32_t stride, float scale, int32_t stride_h, int32_t bias_stride_h, int32_t HEAD_DIM,
                         uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);

/* The hand-written MSL FA2 kernels of the reference's benchmarks:
 *   bench/bench_flash_attention.py:142-149      flash_attention_fwd
 *   bench/bench_flash_attention_opt.py:145-152  flash_attention_opt
 *   bench/bench_fa2_d128.py:116-123             flash_attention_d128
 * each (Q, K, V, O, N, d_head, scale) with Q, K, V, O single-head [N, d]
 * contiguous in one io_type: fp16 when use_half = 1, fp32 when use_half = 0.
 * Constexprs are the MSL generator's parameters (BM, BN, d, THREADS,
 * use_half); d_head must equal d (64 or 128; 128 for flash_attention_d128).
 * Reference grid: (N / BM, 1, 1) with N a multiple of BM; THREADS (1024 in
 * the reference) is accepted and ignored. fp32 operands are rounded to fp16
 * for the tensor cores (the stream's input workspace holds the copies); O is
 * written in io_type. The MSL flash_attention_fwd is exported with an _msl
 * suffix because the TTIR kernel of the same name is exported above. */
NESO_API int neso_flash_attention_fwd_msl(const void* Q, const void* K, const void* V, void* O, int32_t N,
                                          int32_t d_head, float scale, int32_t BM, int32_t BN, int32_t d,
                                          int32_t THREADS, int32_t use_half, uint32_t grid_x, uint32_t grid_y,
                                          uint32_t grid_z, neso_stream_t stream);
NESO_API int neso_flash_attention_opt(const void* Q, const void* K, const void* V, void* O, int32_t N, int32_t d_head,
                                      float scale, int32_t BM, int32_t BN, int32_t d, int32_t THREADS,
                                      int32_t use_half, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                                      neso_stream_t stream);
NESO_API int neso_flash_attention_d128(const void* Q, const void* K, const void* V, void* O, int32_t N,
                                       int32_t d_head, float scale, int32_t BM, int32_t BN, int32_t d,
                                       int32_t THREADS, int32_t use_half, uint32_t grid_x, uint32_t grid_y,
                                       uint32_t grid_z, neso_stream_t stream);

/* Extension (no reference kernel): multi-head FA2 forward over contiguous
 * [B, H, S, D] fp16 Q/K/V with fp32 O [B, H, S, D]. D in {64, 128}, any S >= 1.
 * causal != 0 masks keys j > i. */
NESO_API int neso_fa2_fwd(const void* Q, const void* K, const void* V, float* O, int32_t B, int32_t H, int32_t S, int32_t D,
                 float scale, int32_t causal, neso_stream_t stream);

/* Extension (no reference kernel; nearest is tests/test_rel_pos_fa2.py, whose
 * index is T-1-i+j on a dense table): logits s_ij = (q_i . k_j) * scale +
 * table[h, i - j + S - 1] with an fp32 table [H, 2S - 1]; fp32 O [B, H, S, D]. */
NESO_API int neso_fa2_fwd_relpos_table(const void* Q, const void* K, const void* V, const float* table, float* O, int32_t B,
                              int32_t H, int32_t S, int32_t D, float scale, int32_t causal, neso_stream_t stream);

/* --------------------------------------------------------------- matmul -- */
/* tests/test_aot.py:70-99 (tests/test_triton_jit.py:229-254 for the fp32-C form)
 *   matmul_kernel(a, b, c, M, N, K, stride_am, stride_ak, stride_bk, stride_bn,
 *                 stride_cm, stride_cn, BLOCK_M, BLOCK_N, BLOCK_K)
 * a fp16 [M, K], b fp16 [K, N], c fp32 [M, N]; fp32 accumulation. Unit inner
 * strides (stride_ak = stride_bn = stride_cn = 1), row strides multiples of 8.
 * Reference grid: (cdiv(M, BLOCK_M), cdiv(N, BLOCK_N), 1). */
NESO_API int neso_matmul_kernel(const void* a, const void* b, float* c, int32_t M, int32_t N, int32_t K, int32_t stride_am,
                       int32_t stride_ak, int32_t stride_bk, int32_t stride_bn, int32_t stride_cm, int32_t stride_cn,
                       int32_t BLOCK_M, int32_t BLOCK_N, int32_t BLOCK_K, uint32_t grid_x, uint32_t grid_y,
                       uint32_t grid_z, neso_stream_t stream);

/* bench/bench_matmul.py:79-81 (TTIR) / bench/bench_matmul_opt.py:129-139 (MSL)
 *   matmul_kernel(a, b, c, K, stride_am, stride_bk, stride_cm), constexpr BM, BN.
 * No M/N arguments: M = grid_x * BM, N = grid_y * BN (the reference has no masks). */
NESO_API int neso_matmul_tiled(const void* a, const void* b, float* c, int32_t K, int32_t stride_am, int32_t stride_bk,
                      int32_t stride_cm, int32_t BM, int32_t BN, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                      neso_stream_t stream);

/* ------------------------------------------------------ quantized matmul -- */
/* tests/test_quantized_matmul.py:67-167
 *   w8a16_matmul(A, B, C, K, stride_am, stride_bk, stride_cm), constexpr BM, BN, BK.
 * A fp16 [M, K], B int8 [K, N], C fp32 [M, N]; C = A . f16(B).
 * M = grid_x * BM, N = grid_y * BN (no masks in the reference). */
NESO_API int neso_w8a16_matmul(const void* A, const int8_t* B, float* C, int32_t K, int32_t stride_am, int32_t stride_bk,
                      int32_t stride_cm, int32_t BM, int32_t BN, int32_t BK, uint32_t grid_x, uint32_t grid_y,
                      uint32_t grid_z, neso_stream_t stream);

/* tests/test_quantized_matmul.py:181-283
 *   w8a16_scaled_matmul(A, B, C, scale, K, stride_am, stride_bk, stride_cm)
 * C[m, n] = (sum_k A[m, k] * B[k, n]) * f32(scale[n]); scale fp16 [N]. */
NESO_API int neso_w8a16_scaled_matmul(const void* A, const int8_t* B, float* C, const void* scale, int32_t K,
                             int32_t stride_am, int32_t stride_bk, int32_t stride_cm, int32_t BM, int32_t BN,
                             int32_t BK, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);

/* tests/test_advanced12.py:19-48
 *   w8a16_matmul_kernel(a_ptr, b_int8_ptr, c_ptr, scale_ptr, M, N, K,
 *                       stride_am, stride_ak, stride_bk, stride_bn,
 *                       stride_cm, stride_cn, BLOCK_M, BLOCK_N, BLOCK_K)
 * a fp16 [M, K], b int8 [K, N], c fp32 [M, N], scale_ptr one fp32 value:
 * c = (a . f16(b)) * scale_ptr[0], fp32 accumulation. Unit inner strides,
 * stride_am a multiple of 8, stride_bk a multiple of 16. Reference grid:
 * (cdiv(M, BLOCK_M), cdiv(N, BLOCK_N), 1). */
NESO_API int neso_w8a16_matmul_kernel(const void* a_ptr, const int8_t* b_int8_ptr, float* c_ptr,
                                      const float* scale_ptr, int32_t M, int32_t N, int32_t K, int32_t stride_am,
                                      int32_t stride_ak, int32_t stride_bk, int32_t stride_bn, int32_t stride_cm,
                                      int32_t stride_cn, int32_t BLOCK_M, int32_t BLOCK_N, int32_t BLOCK_K,
                                      uint32_t grid_x, uint32_t grid_y, uint32_t grid_z, neso_stream_t stream);
/* The same kernel with b held in an int32 tensor, as the reference's test
 * passes it (tests/test_advanced12.py:184-186): values in [-128, 127]
 * (others saturate), stride_bk in int32 elements, N a multiple of 16. The
 * weights are narrowed to int8 in the stream's input workspace first. */
NESO_API int neso_w8a16_matmul_kernel_i32(const void* a_ptr, const int32_t* b_int8_ptr, float* c_ptr,
                                          const float* scale_ptr, int32_t M, int32_t N, int32_t K, int32_t stride_am,
                                          int32_t stride_ak, int32_t stride_bk, int32_t stride_bn,
                                          int32_t stride_cm, int32_t stride_cn, int32_t BLOCK_M, int32_t BLOCK_N,
                                          int32_t BLOCK_K, uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                                          neso_stream_t stream);

/* Extension with explicit sizes (any M >= 1): Y fp32 [M, N] = X fp16 [M, K] .
 * (W int8 [K, N] * scale fp16 [N]); scale may be NULL (unscaled W8A16).
 * Row-major, contiguous. N and K multiples of 16. */
NESO_API int neso_w8a16_matmul_mnk(const void* X, const int8_t* W, const void* scale, float* Y, int32_t M, int32_t N,
                          int32_t K, neso_stream_t stream);

/* Extension (no reference kernel; group semantics follow the grouped dequant
 * of tests/test_advanced12.py:69-84): packed int4, group 128, symmetric.
 * Wq uint8 [K/2, N]: byte (k/2, n) holds k even in bits 0-3 and k odd in bits
 * 4-7, two's-complement nibbles in [-8, 7]; scales fp16 [K/128, N].
 * Y fp32 [M, N] = sum_g scales[g, n] * sum_{k in g} X[m, k] * q[k, n].
 * K a multiple of 128, N a multiple of 16. */
NESO_API int neso_w4a16_g128_matmul(const void* X, const uint8_t* Wq, const void* scales, float* Y, int32_t M, int32_t N,
                           int32_t K, neso_stream_t stream);

/* No counterpart in the reference: an allocation-free form of
 * neso_w8a16_matmul_mnk for callers that cannot call cudaMalloc (for example
 * code running inside a host allocator callback, a pre-reserved memory pool
 * manager, or an environment whose device memory is fully budgeted before
 * launch). Same arguments and result (K = 0 writes zeros). It always runs the
 * tensor-core kernel (decode batches of M <= 4 do not take the GEMV path,
 * which keeps per-launch counters in allocated memory). Its split-K scratch is
 * a fixed array of 2^20 floats (4 MiB) compiled into the library, which every
 * GPU that loads the library keeps until the process exits; the K split is
 * chosen among those whose partial sums (splits x M x N floats) fit it, down
 * to no split at all, so no problem is refused for want of scratch. The first
 * call on a device resolves the array's address and should come before any
 * stream capture. All calls on a device share the array: calls that overlap
 * on the GPU (different streams, or concurrent host threads) race and must be
 * serialised by the caller. A timed-out device wait inside it is reported by
 * neso_device_status until neso_clear_device_status. */
NESO_API int neso_w8a16_matmul_mnk_noalloc(const void* X, const int8_t* W, const void* scale, float* Y, int32_t M,
                                           int32_t N, int32_t K, neso_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NESO_B200_H */
