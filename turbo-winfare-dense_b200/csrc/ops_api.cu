// Kernel-level C ABI (include/g4dense_b200_ops.h): prepared INT4 G64 matrices and the
// verify GEMM on caller-owned device buffers.
#include "g4dense_b200_ops.h"

#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "pgemm.h"
#include "vgemm.h"

namespace {
thread_local std::string g_err;
int fail(cudaError_t e, const char* where) {
    g_err = std::string(where) + ": " + cudaGetErrorString(e);
    return (int)e;
}
int fail_msg(const char* msg) {
    g_err = msg;
    return (int)cudaErrorInvalidValue;
}
}  // namespace

namespace {
// Library-owned split-K scratch of g4b_qmat_run_noalloc: 8 MiB of partial slots and one
// arrival counter per 256-row group. Static device memory is part of the module image, so
// using it allocates nothing at call time.
constexpr size_t kNoAllocPartFloats = (size_t)2 << 20;  // 8 MiB
constexpr int kNoAllocCounters = 4096;                 // N <= 4096 * 256 rows
__device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
__device__ __align__(256) unsigned g_noalloc_cnt[kNoAllocCounters];

struct NoAllocScratch {
    float* part = nullptr;
    unsigned* cnt = nullptr;
};
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
NoAllocScratch g_noalloc[kMaxDevices];  // symbol addresses per device ordinal

// Looks up the device addresses of the static scratch on `dev` (the current device) and caches
// them. The first lookup on a device loads the module holding the arrays, which reserves their
// device memory; g4b_qmat_create calls this so that the no-alloc call itself never does. A
// later lookup allocates nothing and refreshes the cache (the addresses are only valid for the
// primary context they were taken in).
cudaError_t noalloc_scratch_setup(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void* part = nullptr;
    void* cnt = nullptr;
    cudaError_t e;
    if ((e = cudaGetSymbolAddress(&part, g_noalloc_part)) != cudaSuccess) return e;
    if ((e = cudaGetSymbolAddress(&cnt, g_noalloc_cnt)) != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    g_noalloc[dev].part = static_cast<float*>(part);
    g_noalloc[dev].cnt = static_cast<unsigned*>(cnt);
    return cudaSuccess;
}
}  // namespace

struct g4b_qmat {
    int N, K, ktiles, n_wrg, n_crg;
    void* w;          // repacked weights
    void* bfrag;      // B fragments for one input of up to 16 rows
    float* part;      // split-K partials
    unsigned* cnt;    // split-K arrival counters [n_crg], zero between launches
    int max_slots;    // slots per row group sized for every M
    int* err;         // device error word of the bounded waits
    // prefill GEMM (17..128 rows): its weight layout, split-K slots and tile counters
    void* pw;
    float* ppart;
    unsigned* pcnt;
    int n_tiles, pmax_slots;
    int dev;          // device the matrix lives on
};

extern "C" {

const char* g4b_last_error(void) { return g_err.c_str(); }

int g4b_qmat_create(const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K, void* stream,
                    g4b_qmat** out) {
    if (!out || !W || !S || !B || N <= 0 || K <= 0 || K % 64) return fail_msg("g4b_qmat_create: bad arguments");
    cudaStream_t st = (cudaStream_t)stream;
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return fail(e0, "g4b_qmat_create: cudaGetDevice");
    // Loads the module that holds g4b_qmat_run_noalloc's static scratch on this device now,
    // while allocating is allowed: under lazy module loading the first symbol lookup reserves
    // that module's device memory.
    if ((e0 = noalloc_scratch_setup(dev)) != cudaSuccess) return fail(e0, "g4b_qmat_create: static scratch set-up");
    auto* q = new g4b_qmat{};
    q->dev = dev;
    q->N = N;
    q->K = K;
    q->ktiles = vgemm_ktiles(K);
    q->n_wrg = (N + 63) / 64;
    q->n_crg = vgemm_n_crg(N);
    cudaError_t e;
    if ((e = cudaMalloc(&q->w, vgemm_weight_bytes(N, K))) != cudaSuccess) { delete q; return fail(e, "cudaMalloc(weights)"); }
    if ((e = g4b_repack(W, S, B, N, K, q->w, st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "repack"); }
    const int Kp = q->ktiles * 128;
    if ((e = cudaMalloc(&q->bfrag, g4b::bfrag_capacity(Kp))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(bfrag)"); }
    q->max_slots = vgemm_plan_slots(q->n_crg, q->ktiles);
    const size_t part_bytes = (size_t)q->n_crg * q->max_slots * g4b::kMaxM * 256 * sizeof(float);
    if ((e = cudaMalloc(&q->part, part_bytes)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(part)"); }
    if ((e = cudaMalloc(&q->cnt, q->n_crg * sizeof(unsigned))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(cnt)"); }
    if ((e = cudaMemsetAsync(q->cnt, 0, q->n_crg * sizeof(unsigned), st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "memset"); }
    if ((e = cudaMalloc(&q->err, sizeof(int))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(err)"); }
    q->n_tiles = pgemm_n_tiles(N);
    q->pmax_slots = pgemm_max_slots(q->n_tiles, K / 64, pgemm_grid(q->n_tiles, K / 64));
    if ((e = cudaMalloc(&q->pw, pgemm_weight_bytes(N, K))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(prefill weights)"); }
    if ((e = pgemm_repack(W, S, B, N, K, q->pw, st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "prefill repack"); }
    if ((e = cudaMalloc(&q->ppart, pgemm_part_floats(q->n_tiles, q->pmax_slots) * sizeof(float))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(prefill part)"); }
    if ((e = cudaMalloc(&q->pcnt, q->n_tiles * sizeof(unsigned))) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "cudaMalloc(prefill cnt)"); }
    if ((e = cudaMemsetAsync(q->pcnt, 0, q->n_tiles * sizeof(unsigned), st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "memset"); }
    if ((e = cudaMemsetAsync(q->err, 0, sizeof(int), st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "memset"); }
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) { g4b_qmat_destroy(q); return fail(e, "g4b_qmat_create"); }
    *out = q;
    return 0;
}

void g4b_qmat_destroy(g4b_qmat* q) {
    if (!q) return;
    cudaFree(q->w);
    cudaFree(q->bfrag);
    cudaFree(q->part);
    cudaFree(q->cnt);
    cudaFree(q->err);
    cudaFree(q->pw);
    cudaFree(q->ppart);
    cudaFree(q->pcnt);
    delete q;
}

int g4b_qmat_prepare_input(g4b_qmat* q, const float* x, int ldx, int M, void* stream) {
    if (!q || !x || M < 1 || M > g4b::kPrefillRows || ldx < q->K)
        return fail_msg("g4b_qmat_prepare_input: bad arguments");
    cudaError_t e = g4b_bfrag_from_f32(x, ldx, M, q->K, q->bfrag, (cudaStream_t)stream, false);
    return e == cudaSuccess ? 0 : fail(e, "bfrag_from_f32");
}

static PartView qmat_view(const g4b_qmat* q, int M) {
    PartView v;
    v.part = q->part;
    v.max_slots = q->max_slots;
    v.n_crg = q->n_crg;
    v.ktiles = q->ktiles;
    v.grid = vgemm_grid(M, q->n_crg, q->ktiles);
    return v;
}

static VgemmParams qmat_params(g4b_qmat* q, int M) {
    const g4b::BFragView v = g4b::bfrag_view(q->bfrag, q->ktiles * 128, M);
    VgemmParams p{};
    p.w = q->w;
    p.bfrag = v.frag;
    p.gsum = v.gsum;
    p.out = qmat_view(q, M);
    p.N = q->N;
    p.M = M;
    p.n_wrg = q->n_wrg;
    p.err = q->err;
    return p;
}

// GEMM kernel without its split-K sum: leaves the partials in the matrix's workspace.
int g4b_qmat_run_partial(g4b_qmat* q, int M, void* stream) {
    if (!q || M < 1 || M > g4b::kMaxM) return fail_msg("g4b_qmat_run_partial: bad arguments");
    cudaError_t e = vgemm_launch(qmat_params(q, M), (cudaStream_t)stream, false);
    return e == cudaSuccess ? 0 : fail(e, "vgemm_launch");
}

int g4b_qmat_run(g4b_qmat* q, int M, float* out, int ldo, void* stream) {
    if (!q || !out || M < 1 || M > g4b::kPrefillRows || ldo < q->N) return fail_msg("g4b_qmat_run: bad arguments");
    if (M > g4b::kMaxM) {
        PgemmParams pp{};
        pp.w = q->pw;
        pp.act = q->bfrag;
        pp.g_layout = q->ktiles * 2;
        pp.y = out;
        pp.ldy = ldo;
        pp.part = q->ppart;
        pp.cnt = q->pcnt;
        pp.N = q->N;
        pp.K = q->K;
        pp.M = M;
        pp.n_tiles = q->n_tiles;
        pp.max_slots = q->pmax_slots;
        pp.err = q->err;
        cudaError_t e = pgemm_launch(pp, (cudaStream_t)stream, false);
        return e == cudaSuccess ? 0 : fail(e, "pgemm_launch");
    }
    VgemmParams p = qmat_params(q, M);
    p.y = out;
    p.ldy = ldo;
    p.cnt = q->cnt;
    cudaError_t e = vgemm_launch(p, (cudaStream_t)stream, false);
    return e == cudaSuccess ? 0 : fail(e, "vgemm_launch");
}

// ---------------------------------------------------------------- allocation-free run


int g4b_qmat_run_noalloc(g4b_qmat* q, int M, float* out, int ldo, void* stream) {
    if (!q || !out || ldo < q->N) return fail_msg("g4b_qmat_run_noalloc: bad arguments");
    if (M < 1 || M > g4b::kMaxM)
        return fail_msg("g4b_qmat_run_noalloc: M must be 1..16 (the verify GEMM only; 17..128 rows need "
                        "g4b_qmat_run's tensor-core path and its allocated workspace)");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(e, "g4b_qmat_run_noalloc: cudaGetDevice");
    if (dev != q->dev) return fail_msg("g4b_qmat_run_noalloc: the current device is not the matrix's device");
    NoAllocScratch sc;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        sc = g_noalloc[dev];
    }
    if (!sc.part) return fail_msg("g4b_qmat_run_noalloc: static scratch not set up on this device");
    VgemmParams p = qmat_params(q, M);
    // Exactly the slots this launch needs (the matrix's own workspace is sized for every M).
    const int slots = vgemm_max_slots(p.out.grid, q->n_crg, q->ktiles);
    const size_t need = (size_t)q->n_crg * slots * g4b::kMaxM * 256;
    if (need > kNoAllocPartFloats || q->n_crg > kNoAllocCounters) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "g4b_qmat_run_noalloc: this matrix needs %.1f MiB of split-K scratch at M = %d (%d row groups x "
                      "%d slots); the static buffer holds 8 MiB and %d row groups -- use g4b_qmat_run",
                      need * 4.0 / (1 << 20), M, q->n_crg, slots, kNoAllocCounters);
        return fail_msg(msg);
    }
    p.out.part = sc.part;
    p.out.max_slots = slots;
    p.y = out;
    p.ldy = ldo;
    p.cnt = sc.cnt;
    const cudaStream_t st = (cudaStream_t)stream;
    // The arrival counters must start at zero; a complete launch leaves them at zero, a failed
    // one may not, so they are cleared on the stream first.
    if ((e = cudaMemsetAsync(sc.cnt, 0, (size_t)q->n_crg * sizeof(unsigned), st)) != cudaSuccess)
        return fail(e, "g4b_qmat_run_noalloc: clearing counters");
    e = vgemm_launch(p, st, false);
    return e == cudaSuccess ? 0 : fail(e, "g4b_qmat_run_noalloc: vgemm_launch");
}

int g4b_qmat_gemm(g4b_qmat* q, const float* x, int ldx, int M, float* out, int ldo, void* stream) {
    int rc = g4b_qmat_prepare_input(q, x, ldx, M, stream);
    return rc ? rc : g4b_qmat_run(q, M, out, ldo, stream);
}

int g4b_qmat_info(const g4b_qmat* q, int* out4) {
    if (!q || !out4) return fail_msg("g4b_qmat_info: bad arguments");
    out4[0] = q->N;
    out4[1] = q->K;
    out4[2] = vgemm_grid(5, q->n_crg, q->ktiles);
    out4[3] = q->max_slots;
    return 0;
}

int g4b_gemv_int8(const uint8_t* W, const uint16_t* S, const uint16_t* B, const float* x, float* out, int rows,
                  int K, void* stream) {
    if (!W || !S || !B || !x || !out || rows <= 0 || K <= 0 || K % 64)
        return fail_msg("g4b_gemv_int8: bad arguments (K must be a positive multiple of 64)");
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x)) & 15)
        return fail_msg("g4b_gemv_int8: W and x must be 16-byte aligned");
    const cudaError_t e = g4b::gemv_int8_launch(W, S, B, x, out, rows, K, (cudaStream_t)stream);
    return e == cudaSuccess ? 0 : fail(e, "g4b_gemv_int8");
}

int g4b_attn_gate(const float* ctx, const float* gate, float* out, int n, int batch, int ctx_stride, int gate_stride,
                  int out_stride, void* stream) {
    if (!ctx || !gate || !out || n <= 0 || batch < 0 || ctx_stride < n || gate_stride < n || out_stride < n)
        return fail_msg("g4b_attn_gate: bad arguments");
    if (batch == 0) return 0;
    const cudaError_t e =
        g4b::attn_gate_launch(ctx, gate, out, n, batch, ctx_stride, gate_stride, out_stride, (cudaStream_t)stream);
    return e == cudaSuccess ? 0 : fail(e, "g4b_attn_gate");
}

size_t g4b_sample_workspace(void) { return g4b_sample_workspace_bytes(); }

int g4b_sample_token(const float* logits, int vocab, float temperature, float top_p, int top_k, uint64_t seed,
                     void* workspace, uint32_t* out_token, void* stream) {
    if (!logits || !workspace || vocab < 1 || vocab > 262144 || top_k < 0 || top_k > 256 || !(top_p > 0.f) ||
        top_p > 1.f || !(temperature >= 0.f))
        return fail_msg("g4b_sample_token: bad arguments (vocab 1..262144, top_k 0..256, top_p in (0, 1], "
                        "temperature >= 0)");
    const cudaError_t e = g4b_sample_launch(logits, vocab, temperature, top_p, top_k, seed, workspace, out_token,
                                            static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : fail(e, "g4b_sample_token");
}

int g4b_qmat_check_error(g4b_qmat* q) {
    if (!q) return fail_msg("g4b_qmat_check_error: null handle");
    int h = 0;
    cudaError_t e = cudaMemcpy(&h, q->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(e, "g4b_qmat_check_error");
    if (h) return fail_msg("INT4 GEMM: a bounded wait gave up (weights or fragments never arrived)");
    return 0;
}

}  // extern "C"
