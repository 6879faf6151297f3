/* Kernel-level C ABI of the B200 speculative-decode library (libg4dense_b200.so).
 *
 * These entry points expose single hot-path operators on caller-owned DEVICE buffers, so a
 * host that already manages CUDA memory can bind them the way the reference's host binds its
 * compute shaders. All pointers are device pointers unless stated otherwise; `stream` is a
 * cudaStream_t (NULL = legacy default stream). Functions return 0 on success or a CUDA error
 * code, with a message in g4b_last_error() (thread-local), mirroring the reference's
 * g4dense_engine_last_error convention (src/c_api.cpp:28-31).
 */
#ifndef G4DENSE_B200_OPS_H
#define G4DENSE_B200_OPS_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4B_API __attribute__((visibility("default")))

G4B_API const char* g4b_last_error(void);

/* A prepared INT4 G64 affine matrix. Replaces the reference's weight binding for
 * GemvInt4 / GemmInt4Batch (shaders/GemvInt4.hlsl:24-25, shaders/GemmInt4Batch.hlsl:296-301):
 * W [N][K/8] u32 (nibble c%8 of word c/8, low nibble first), S and B [N][K/64] bf16, all in
 * the container's row-major layout. The matrix is repacked once into the B200 streaming
 * layout; the source buffers may be freed afterwards. K must be a multiple of 64. */
typedef struct g4b_qmat g4b_qmat;
G4B_API int g4b_qmat_create(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K,
                            void* stream, g4b_qmat** out);
G4B_API void g4b_qmat_destroy(g4b_qmat* q);

/* out[m][n] = sum_k (q[n][k] * s + b) * x[m][k] for m < M <= 128: the batched INT4 GEMM
 * (shaders/GemmInt4Batch.hlsl:64-143; M = 1 is GemvInt4, shaders/GemvInt4.hlsl:31-54).
 * M <= 16 runs the HBM-streaming verify GEMM; 17 <= M <= 128 (prefill chunks) the tcgen05
 * tensor-core GEMM. x is fp32 [M][ldx], out fp32 [M][ldo]. Launches two kernels: activation
 * preparation and the GEMM. Calls on one matrix must be stream-ordered (they share the
 * matrix's workspace). */
G4B_API int g4b_qmat_gemm(g4b_qmat* q, const float* x, int ldx, int M, float* out, int ldo, void* stream);
/* The two halves of g4b_qmat_gemm, for timing the GEMM kernel alone. */
G4B_API int g4b_qmat_prepare_input(g4b_qmat* q, const float* x, int ldx, int M, void* stream);
G4B_API int g4b_qmat_run(g4b_qmat* q, int M, float* out, int ldo, void* stream);
/* The verify GEMM kernel (M <= 16) without its in-kernel split-K sum, leaving the partials in
 * the matrix's workspace (for timing the weight stream alone). */
G4B_API int g4b_qmat_run_partial(g4b_qmat* q, int M, void* stream);
/* g4b_qmat_run for M = 1..16 (the verify GEMM only) without any allocation: the same kernel,
 * grid and slot order (bit-identical output), but the split-K scratch -- partial slots and
 * per-row-group arrival counters -- is a fixed static device buffer inside the library (8 MiB of
 * slots, 4096 row groups) instead of the matrix's own workspace. No counterpart in the reference,
 * whose shaders take their scratch from buffers bound by the host. For callers that must not
 * allocate device memory at call time: code running inside a caching allocator's callbacks or on
 * a device whose memory a pool has fully reserved, and latency-sensitive loops where
 * cudaMalloc/cudaFree would synchronize the device.
 *   - Rejects (non-zero return, message in g4b_last_error) M outside 1..16 (17..128 rows need
 *     g4b_qmat_run's tensor-core path), and a matrix whose launch at this M needs more than
 *     8 MiB of slots or more than 4096 row groups (N > 1048576).
 *   - The static buffer lives in a module that CUDA loads lazily; loading it reserves its
 *     device memory. g4b_qmat_create loads it on the matrix's device (it allocates anyway), so
 *     this call itself allocates nothing. It must run on the device the matrix was created on.
 *   - The counters are cleared on `stream` before the launch.
 *   - The scratch is shared by every caller on a device: overlapping calls (other streams,
 *     other threads) race and must be ordered by the caller.
 *   - Not valid across a device or primary-context reset: the cached scratch address dies
 *     with the context. Create the matrix again after a reset. */
G4B_API int g4b_qmat_run_noalloc(g4b_qmat* q, int M, float* out, int ldo, void* stream);
/* Synchronizes and reports whether any launch on q hit a bounded-wait timeout. */
G4B_API int g4b_qmat_check_error(g4b_qmat* q);
/* INT8 G64 affine GEMV, the reference's GemvInt8 (shaders/GemvInt8.hlsl:13-33, row dot
 * shaders/Common.hlsli:225-269): out[r] = sum_k (W[r][k] * s + b) * x[k] for r < rows, with W
 * [rows][K] u8, S and B [rows][K/64] bf16, x [K] fp32, out [rows] fp32. K a multiple of 64; W and
 * x 16-byte aligned. */
G4B_API int g4b_gemv_int8(const uint8_t* W, const uint16_t* S, const uint16_t* B, const float* x, float* out,
                          int rows, int K, void* stream);
/* Attention output gate, the reference's AttnGate (shaders/AttnGate.hlsl:15-32):
 * out[m][c] = ctx[m][c] * sigmoid(gate[m][c]) for c < n, m < batch; strides in floats. */
G4B_API int g4b_attn_gate(const float* ctx, const float* gate, float* out, int n, int batch, int ctx_stride,
                          int gate_stride, int out_stride, void* stream);
/* Token sampling on a device logits row, the reference's sample_token (src/sampling.cpp:92-169):
 * greedy argmax (ties to the lowest index) when temperature <= 0; otherwise the top_k (or 256)
 * largest logits, a top-p cut measured against the full-vocabulary softmax, and a
 * temperature-scaled draw with the xorshift64* generator seeded with `seed` (the caller derives it
 * as the reference's seed_for does, src/sampling.cpp:63-72). logits: fp32 [vocab] device memory,
 * vocab <= 262144; top_k 0..256 (0 = 256-wide shortlist); top_p in (0, 1]. `workspace` is
 * g4b_sample_workspace() bytes of device memory, used by one stream at a time; the token is
 * written to out_token (device memory). Two kernel launches. */
G4B_API size_t g4b_sample_workspace(void);
G4B_API int g4b_sample_token(const float* logits, int vocab, float temperature, float top_p, int top_k,
                             uint64_t seed, void* workspace, uint32_t* out_token, void* stream);
/* out4 = {N, K, grid CTAs at M=5, split-K slots per row group} */
G4B_API int g4b_qmat_info(const g4b_qmat* q, int* out4);

#ifdef __cplusplus
}
#endif
#endif
