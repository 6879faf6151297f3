/* CPU restatement of the reference's speculative-decode path. TEST INFRASTRUCTURE ONLY.
 * See g4d_oracle.h for the contract. Build: make -C oracle restate (gcc -O2, no FMA
 * contraction, so the arithmetic order matches src/cpu_reference.cpp exactly). */
#define _GNU_SOURCE
#include "g4d_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static __thread char g_err[512];
static void set_err(const char* msg) { snprintf(g_err, sizeof g_err, "%s", msg); }
const char* g4o_last_error(void) { return g_err; }

/* ------------------------------------------------------------------ numerics helpers */

/* src/cpu_reference.cpp:39-44 */
float g4o_bf16_to_f32(uint16_t v) {
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t g4o_f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float g4o_round_bf16(float f) { return g4o_bf16_to_f32(g4o_f32_to_bf16_rne(f)); }

/* Round-trip through IEEE FP16, src/cpu_reference.cpp:51-84 (subnormal halves flush to
 * signed zero on the way in, exactly as the reference does). */
float g4o_round_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    uint32_t man = x & 0x7FFFFFu;
    uint16_t h;
    if (e <= 0) h = (uint16_t)sign;
    else if (e >= 31) h = (uint16_t)(sign | 0x7C00u);
    else {
        const uint32_t round_bit = (man >> 12) & 1u;
        const uint32_t sticky = (man & 0xFFFu) != 0u;
        uint32_t v = sign | ((uint32_t)e << 10) | (man >> 13);
        if (round_bit && (sticky || (v & 1u))) ++v;
        h = (uint16_t)v;
    }
    const uint32_t s2 = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e2 = (h >> 10) & 0x1Fu;
    uint32_t m2 = h & 0x3FFu;
    uint32_t bits;
    if (e2 == 0) {
        if (m2 == 0) bits = s2;
        else {
            e2 = 1;
            while ((m2 & 0x400u) == 0) { m2 <<= 1; --e2; }
            m2 &= 0x3FFu;
            bits = s2 | ((e2 + 127 - 15) << 23) | (m2 << 13);
        }
    } else if (e2 == 0x1Fu) bits = s2 | 0x7F800000u | (m2 << 13);
    else bits = s2 | ((e2 + 127 - 15) << 23) | (m2 << 13);
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* src/cpu_reference.cpp:87-91 and shaders/Common.hlsli:145-149 */
float g4o_gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    float inner = k * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* Dequantize affine INT4 G64 rows to fp32, src/cpu_reference.cpp:94-126. */
static void dequant_int4(const uint32_t* W, const uint16_t* S, const uint16_t* B, uint32_t rows,
                         uint32_t cols, float* out) {
    const uint32_t gpr = cols / 64, pc = cols / 8;
    for (uint32_t r = 0; r < rows; ++r) {
        const uint32_t* rw = W + (size_t)r * pc;
        const uint16_t* rs = S + (size_t)r * gpr;
        const uint16_t* rb = B + (size_t)r * gpr;
        float* o = out + (size_t)r * cols;
        for (uint32_t c = 0; c < cols; ++c) {
            const uint32_t q = (rw[c / 8] >> ((c % 8) * 4)) & 0xFu;
            o[c] = (float)q * g4o_bf16_to_f32(rs[c / 64]) + g4o_bf16_to_f32(rb[c / 64]);
        }
    }
}

/* Sequential fp32 dot, the order of gemv in src/cpu_reference.cpp:129-138. */
static void gemv_f32(const float* W, const float* in, uint32_t rows, uint32_t cols, float* out) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float* row = W + (size_t)r * cols;
        float s = 0.0f;
        for (uint32_t c = 0; c < cols; ++c) s += row[c] * in[c];
        out[r] = s;
    }
}

/* GemmInt4Batch semantics (shaders/GemmInt4Batch.hlsl:64-143, Common.hlsli:163-222):
 * out[m][r] = sum_c (q*s+b) * x[m][c], summed in column order. */
void g4o_int4_gemm(const uint32_t* W, const uint16_t* S, const uint16_t* B, uint32_t rows,
                   uint32_t cols, const float* x, uint32_t M, float* out) {
    float* row = (float*)malloc(sizeof(float) * cols);
    for (uint32_t r = 0; r < rows; ++r) {
        dequant_int4(W + (size_t)r * (cols / 8), S + (size_t)r * (cols / 64),
                     B + (size_t)r * (cols / 64), 1, cols, row);
        for (uint32_t m = 0; m < M; ++m) {
            const float* xm = x + (size_t)m * cols;
            float s = 0.0f;
            for (uint32_t c = 0; c < cols; ++c) s += row[c] * xm[c];
            out[(size_t)m * rows + r] = s;
        }
    }
    free(row);
}

/* GemvInt8 (shaders/GemvInt8.hlsl:13-33, Common.hlsli:225-269): one byte per weight, 4 per
 * u32 word low byte first, bf16 scale/bias per 64 columns. */
void g4o_int8_gemv(const uint32_t* W, const uint16_t* S, const uint16_t* B, uint32_t rows,
                   uint32_t cols, const float* x, float* out) {
    const uint32_t gpr = cols / 64;
    for (uint32_t r = 0; r < rows; ++r) {
        const uint8_t* rw = (const uint8_t*)(W + (size_t)r * (cols / 4));
        float s = 0.0f;
        for (uint32_t c = 0; c < cols; ++c) {
            const float w = (float)rw[c] * g4o_bf16_to_f32(S[(size_t)r * gpr + c / 64]) +
                            g4o_bf16_to_f32(B[(size_t)r * gpr + c / 64]);
            s += w * x[c];
        }
        out[r] = s;
    }
}

/* Attention output gate: out = ctx * (1 / (1 + exp(-gate))) (src/cpu_reference.cpp:550-556,
 * shaders/AttnGate.hlsl:15-32). */
void g4o_attn_gate(const float* ctx, const float* gate, float* out, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        const float sig = 1.0f / (1.0f + expf(-gate[i]));
        out[i] = ctx[i] * sig;
    }
}

/* rms_norm, src/cpu_reference.cpp:141-150 (w == NULL: rms_norm_no_scale, :153-162). */
static void rms_norm_f(const float* x, const float* w, uint32_t n, float eps, float* out) {
    float ss = 0.0f;
    for (uint32_t i = 0; i < n; ++i) ss += x[i] * x[i];
    const float rms = 1.0f / sqrtf((ss / (float)n) + eps);
    for (uint32_t i = 0; i < n; ++i) out[i] = w ? x[i] * rms * w[i] : x[i] * rms;
}

void g4o_rmsnorm(const float* x, const uint16_t* w_bf16, uint32_t n, float eps, float* out) {
    float* w = NULL;
    if (w_bf16) {
        w = (float*)malloc(sizeof(float) * n);
        for (uint32_t i = 0; i < n; ++i) w[i] = g4o_bf16_to_f32(w_bf16[i]);
    }
    rms_norm_f(x, w, n, eps, out);
    free(w);
}

/* Two-pass softmax attention of src/cpu_reference.cpp:504-548, for one query row. */
static void attend_row(const float* qh_vec, const float* K, const float* V, uint32_t kvh_count,
                       uint32_t kvh, uint32_t hd, uint32_t start, uint32_t end, float scale,
                       float* scores, float* out_h) {
    const uint32_t win = end - start;
    for (uint32_t t = 0; t < win; ++t) {
        const float* k = K + ((size_t)(start + t) * kvh_count + kvh) * hd;
        float s = 0.0f;
        for (uint32_t d = 0; d < hd; ++d) s += qh_vec[d] * k[d];
        scores[t] = s * scale;
    }
    float mx = -1e9f;
    for (uint32_t t = 0; t < win; ++t) mx = fmaxf(mx, scores[t]);
    float sum = 0.0f;
    for (uint32_t t = 0; t < win; ++t) {
        scores[t] = expf(scores[t] - mx);
        sum += scores[t];
    }
    for (uint32_t t = 0; t < win; ++t) scores[t] /= sum;
    for (uint32_t d = 0; d < hd; ++d) out_h[d] = 0.0f;
    for (uint32_t t = 0; t < win; ++t) {
        const float* v = V + ((size_t)(start + t) * kvh_count + kvh) * hd;
        const float a = scores[t];
        for (uint32_t d = 0; d < hd; ++d) out_h[d] += a * v[d];
    }
}

void g4o_attention(const float* q, const float* K, const float* V, uint32_t M, uint32_t qh,
                   uint32_t kvh, uint32_t hd, uint32_t n_pos, uint32_t window, float scale,
                   float* out) {
    float* scores = (float*)malloc(sizeof(float) * (n_pos + M + 1));
    const uint32_t gqa = qh / kvh;
    for (uint32_t m = 0; m < M; ++m) {
        const uint32_t end = n_pos + m;
        const uint32_t start = (window && end > window) ? end - window : 0;
        for (uint32_t h = 0; h < qh; ++h)
            attend_row(q + ((size_t)m * qh + h) * hd, K, V, kvh, h / gqa, hd, start, end, scale,
                       scores, out + ((size_t)m * qh + h) * hd);
    }
    free(scores);
}

/* ------------------------------------------------------------------ container model */

#pragma pack(push, 1)
typedef struct {
    uint32_t magic, version, quant_type, num_layers, d_model, d_ff, num_q_heads, num_kv_heads,
        head_dim, vocab_size, sliding_window, quant_group_size, scale_dtype, tied_embeddings;
    uint64_t global_layer_mask;
    float rope_theta_local, rope_theta_global, rope_scaling, final_logit_softcapping;
    uint64_t embed_offset, embed_size, lm_head_offset, lm_head_size;
    uint64_t layer_offsets[60];
    uint64_t layer_sizes[60];
    uint8_t payload_sha256[32];
    uint32_t global_head_dim, global_kv_heads;
    uint32_t ple_dim, ple_vocab, num_kv_shared_layers, ple_reserved;
    uint64_t ple_offset, ple_size;
    uint32_t layer_d_ff[60];
    uint32_t arch_type, attn_out_dim;
    float qk_scale_factor, output_multiplier;
    uint8_t reserved[2696];
} g4o_header; /* include/g4dense/format.hpp:26-110 */
#pragma pack(pop)
_Static_assert(sizeof(g4o_header) == 4096, "header layout");

typedef struct {
    const uint32_t* w;
    const uint16_t* s;
    const uint16_t* b;
    uint32_t rows, cols;
    float* cached; /* fp32 copy when cache_dequant */
} qmat;

typedef struct {
    uint32_t hd, qh, kvh, is_global;
    uint32_t ffn;        /* this layer's FFN width (layer_ffn_width, include/g4dense/format.hpp:189-196) */
    uint32_t has_v;      /* 0: V is the raw K (a full-attention layer of a model without per-layer inputs) */
    uint32_t shared;     /* 1: reads the K/V of layer `donor` and has no k, v or k_norm of its own */
    uint32_t donor;
    const uint16_t *in_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm, *q_norm, *k_norm;
    const uint16_t* post_ple_norm; /* per-layer-input models only */
    float layer_scalar;
    qmat q, k, v, o, gate, up, down; /* k/v.rows == 0 where absent */
    qmat ple_gate, ple_proj;         /* [ple_dim][d], [d][ple_dim]; rows == 0 without per-layer inputs */
    float* kcache; /* [max_ctx][kvh*hd]; NULL on a shared layer */
    float* vcache;
} layer_t;

struct g4o_model {
    g4o_header h;
    const uint8_t* base;
    size_t size;
    int kv_mode;
    uint32_t max_ctx, len;
    layer_t* layers;
    qmat embed; /* the tied embedding / LM head */
    const uint16_t* final_norm;
    /* Per-layer inputs (E2B/E4B): the [ple_vocab][L*ple_dim] table, the [L*ple_dim][d]
     * projection of the token embedding and the bf16 [ple_dim] norm of each layer's slice. */
    qmat ple_table, ple_model_proj;
    const uint16_t* ple_norm;
};

/* is_kv_shared_layer / kv_donor_layer, include/g4dense/format.hpp:210-227: the last
 * num_kv_shared_layers layers read the cache of the last non-shared layer of their own type. */
static uint32_t kv_shared_layer(const g4o_header* h, uint32_t l) {
    return h->num_kv_shared_layers && h->num_kv_shared_layers <= h->num_layers &&
           l >= h->num_layers - h->num_kv_shared_layers;
}

static uint32_t kv_donor(const g4o_header* h, uint32_t l) {
    if (!kv_shared_layer(h, l)) return l;
    const uint64_t want = (h->global_layer_mask >> l) & 1ull;
    for (uint32_t d = h->num_layers - h->num_kv_shared_layers; d-- > 0;)
        if (((h->global_layer_mask >> d) & 1ull) == want) return d;
    return 0;
}

/* resolve_layer_geometry, include/g4dense/format.hpp:229-241 */
static void layer_geo(const g4o_header* h, uint32_t l, layer_t* L) {
    L->is_global = (uint32_t)((h->global_layer_mask >> l) & 1ull);
    L->hd = h->head_dim;
    L->qh = h->num_q_heads;
    L->kvh = h->num_kv_heads;
    if (L->is_global) {
        L->hd = h->global_head_dim ? h->global_head_dim : 512u;
        L->kvh = h->global_kv_heads ? h->global_kv_heads : 4u;
    }
}

/* parse_quant_block, src/cpu_reference.cpp:367-381: pad to 16 bytes relative to the layer
 * start, then W [rows][cols/8] u32, scales and biases [rows][cols/64] bf16. */
static const uint8_t* parse_qmat(const uint8_t* layer, const uint8_t* p, uint32_t rows, uint32_t cols,
                                 qmat* q) {
    p += (16u - ((size_t)(p - layer) & 15u)) & 15u;
    const size_t wb = (size_t)rows * (cols / 8) * 4, sb = (size_t)rows * (cols / 64) * 2;
    q->w = (const uint32_t*)p;
    q->s = (const uint16_t*)(p + wb);
    q->b = (const uint16_t*)(p + wb + sb);
    q->rows = rows;
    q->cols = cols;
    q->cached = NULL;
    return p + wb + 2 * sb;
}

/* A quantized matrix stored back to back (W, scales, biases) with no alignment padding, as the
 * per-layer-input block is (tools/convert_hf_to_g4dense.py:180-190). */
static const uint8_t* packed_qmat(const uint8_t* p, uint32_t rows, uint32_t cols, qmat* q) {
    const size_t wb = (size_t)rows * (cols / 8) * 4, sb = (size_t)rows * (cols / 64) * 2;
    q->w = (const uint32_t*)p;
    q->s = (const uint16_t*)(p + wb);
    q->b = (const uint16_t*)(p + wb + sb);
    q->rows = rows;
    q->cols = cols;
    q->cached = NULL;
    return p + wb + 2 * sb;
}

static void cache_q(qmat* q) {
    if (!q->rows) return;
    q->cached = (float*)malloc(sizeof(float) * (size_t)q->rows * q->cols);
    dequant_int4(q->w, q->s, q->b, q->rows, q->cols, q->cached);
}

/* y = W x with the reference's order: full dequant then sequential dot. */
static void qgemv(const qmat* q, const float* x, float* y) {
    if (q->cached) {
        gemv_f32(q->cached, x, q->rows, q->cols, y);
        return;
    }
    float* row = (float*)malloc(sizeof(float) * q->cols);
    for (uint32_t r = 0; r < q->rows; ++r) {
        dequant_int4(q->w + (size_t)r * (q->cols / 8), q->s + (size_t)r * (q->cols / 64),
                     q->b + (size_t)r * (q->cols / 64), 1, q->cols, row);
        float s = 0.0f;
        for (uint32_t c = 0; c < q->cols; ++c) s += row[c] * x[c];
        y[r] = s;
    }
    free(row);
}

g4o_model* g4o_open(const char* path, int kv_mode, uint32_t max_ctx, int cache_dequant) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { set_err("g4o_open: cannot open container"); return NULL; }
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(g4o_header)) {
        close(fd);
        set_err("g4o_open: container too small for header");
        return NULL;
    }
    void* p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) { set_err("g4o_open: mmap failed"); return NULL; }
    g4o_model* m = (g4o_model*)calloc(1, sizeof(g4o_model));
    m->base = (const uint8_t*)p;
    m->size = (size_t)st.st_size;
    memcpy(&m->h, p, sizeof(g4o_header));
    const g4o_header* h = &m->h;
    /* validate_header essentials, src/format.cpp:6-65 */
    if (h->magic != 0x4734444Eu || h->version != 3 || h->num_layers == 0 || h->num_layers > 60 ||
        h->d_model == 0 || h->d_ff == 0 || h->vocab_size == 0 || h->embed_offset % 4096 ||
        h->lm_head_offset % 4096) {
        set_err("g4o_open: invalid header");
        munmap(p, m->size);
        free(m);
        return NULL;
    }
    m->kv_mode = kv_mode;
    m->max_ctx = max_ctx;
    const uint32_t d = h->d_model, f = h->d_ff, V = h->vocab_size;
    m->embed.w = (const uint32_t*)(m->base + h->embed_offset);
    m->embed.s = (const uint16_t*)((const uint8_t*)m->embed.w + (size_t)V * (d / 8) * 4);
    m->embed.b = (const uint16_t*)((const uint8_t*)m->embed.s + (size_t)V * (d / 64) * 2);
    m->embed.rows = V;
    m->embed.cols = d;
    m->embed.cached = NULL;
    m->final_norm = (const uint16_t*)((const uint8_t*)m->embed.b + (size_t)V * (d / 64) * 2);
    const uint32_t ple = h->ple_dim, ple_rows = h->num_layers * h->ple_dim;
    if (ple) {
        /* The per-layer-input block (src/runner.cpp:446-482): the table, the projection, the
         * norm, back to back. */
        if (!h->ple_offset || !h->ple_vocab || ple % 64 || h->ple_offset + h->ple_size > m->size) {
            set_err("g4o_open: invalid per-layer-input block");
            munmap(p, m->size);
            free(m);
            return NULL;
        }
        const uint8_t* b = packed_qmat(m->base + h->ple_offset, h->ple_vocab, ple_rows, &m->ple_table);
        b = packed_qmat(b, ple_rows, d, &m->ple_model_proj);
        m->ple_norm = (const uint16_t*)b;
    }
    (void)f;
    m->layers = (layer_t*)calloc(h->num_layers, sizeof(layer_t));
    for (uint32_t l = 0; l < h->num_layers; ++l) {
        layer_t* L = &m->layers[l];
        layer_geo(h, l, L);
        L->ffn = (l < 60 && h->layer_d_ff[l]) ? h->layer_d_ff[l] : h->d_ff;
        L->shared = kv_shared_layer(h, l);
        L->donor = kv_donor(h, l);
        /* V has its own projection except on full-attention layers of a model without per-layer
         * inputs (src/runner.cpp:351-360). */
        L->has_v = !L->shared && (!L->is_global || ple);
        const uint8_t* lp = m->base + h->layer_offsets[l];
        const uint16_t* n = (const uint16_t*)lp;
        L->in_norm = n;
        L->post_attn_norm = n + d;
        L->pre_ffn_norm = n + 2 * d;
        L->post_ffn_norm = n + 3 * d;
        L->q_norm = n + 4 * d;
        n = L->q_norm + L->hd;
        L->k_norm = L->shared ? NULL : n;
        if (!L->shared) n += L->hd;
        L->layer_scalar = g4o_bf16_to_f32(*n++);
        if (ple) {
            L->post_ple_norm = n;
            n += d;
        }
        const uint8_t* q = (const uint8_t*)n;
        q = parse_qmat(lp, q, L->qh * L->hd, d, &L->q);
        if (!L->shared) q = parse_qmat(lp, q, L->kvh * L->hd, d, &L->k);
        if (L->has_v) q = parse_qmat(lp, q, L->kvh * L->hd, d, &L->v);
        q = parse_qmat(lp, q, d, L->qh * L->hd, &L->o);
        q = parse_qmat(lp, q, L->ffn, d, &L->gate);
        q = parse_qmat(lp, q, L->ffn, d, &L->up);
        q = parse_qmat(lp, q, d, L->ffn, &L->down);
        if (ple) {
            q = parse_qmat(lp, q, ple, d, &L->ple_gate);
            q = parse_qmat(lp, q, d, ple, &L->ple_proj);
        }
        if ((size_t)(q - m->base) > m->size) {
            set_err("g4o_open: layer exceeds file");
            g4o_close(m);
            return NULL;
        }
        if (cache_dequant) {
            cache_q(&L->q); cache_q(&L->k); cache_q(&L->v); cache_q(&L->o);
            cache_q(&L->gate); cache_q(&L->up); cache_q(&L->down);
            cache_q(&L->ple_gate); cache_q(&L->ple_proj);
        }
        if (!L->shared) {
            L->kcache = (float*)malloc(sizeof(float) * (size_t)max_ctx * L->kvh * L->hd);
            L->vcache = (float*)malloc(sizeof(float) * (size_t)max_ctx * L->kvh * L->hd);
        }
    }
    if (cache_dequant) {
        cache_q(&m->embed);
        cache_q(&m->ple_model_proj);
    }
    return m;
}

static void free_q(qmat* q) { free(q->cached); q->cached = NULL; }

void g4o_close(g4o_model* m) {
    if (!m) return;
    for (uint32_t l = 0; l < m->h.num_layers; ++l) {
        layer_t* L = &m->layers[l];
        free_q(&L->q); free_q(&L->k); free_q(&L->v); free_q(&L->o);
        free_q(&L->gate); free_q(&L->up); free_q(&L->down);
        free_q(&L->ple_gate); free_q(&L->ple_proj);
        free(L->kcache);
        free(L->vcache);
    }
    free_q(&m->embed);
    free_q(&m->ple_model_proj);
    free(m->layers);
    munmap((void*)m->base, m->size);
    free(m);
}

void g4o_info(const g4o_model* m, uint32_t* o) {
    const g4o_header* h = &m->h;
    o[0] = h->num_layers; o[1] = h->d_model; o[2] = h->d_ff; o[3] = h->num_q_heads;
    o[4] = h->num_kv_heads; o[5] = h->head_dim; o[6] = h->vocab_size; o[7] = h->sliding_window;
    o[8] = h->global_head_dim; o[9] = h->global_kv_heads;
    o[10] = (uint32_t)(h->global_layer_mask & 0xFFFFFFFFu);
    o[11] = (uint32_t)(h->global_layer_mask >> 32);
}

uint32_t g4o_length(const g4o_model* m) { return m->len; }
void g4o_truncate(g4o_model* m, uint32_t len) { if (len < m->len) m->len = len; }

static float kv_round(int mode, float v) {
    if (mode == G4O_KV_FP16) return g4o_round_f16(v);
    if (mode == G4O_KV_BF16) return g4o_round_bf16(v);
    return v;
}

/* NeoX RoPE on `rotated` pairs (i, i+hd/2), src/cpu_reference.cpp:457-466. */
static void rope(float* x, uint32_t hd, uint32_t rotated, float theta, uint32_t position) {
    const uint32_t half = hd / 2;
    for (uint32_t p = 0; p < rotated; ++p) {
        const float freq = 1.0f / powf(theta, (float)(2 * p) / (float)hd);
        const float angle = (float)position * freq;
        const float c = cosf(angle), s = sinf(angle);
        const float x0 = x[p], x1 = x[p + half];
        x[p] = x0 * c - x1 * s;
        x[p + half] = x0 * s + x1 * c;
    }
}

static void bf16_vec(const uint16_t* src, uint32_t n, float* dst) {
    for (uint32_t i = 0; i < n; ++i) dst[i] = g4o_bf16_to_f32(src[i]);
}

/* forward_single_token, src/cpu_reference.cpp:245-672 (Gemma-4 architecture). */
int g4o_forward(g4o_model* m, uint32_t token, uint32_t pos, float* logits, float* hidden_out) {
    const g4o_header* h = &m->h;
    if (pos != m->len) { set_err("g4o_forward: position must equal the cache length"); return -1; }
    if (pos >= m->max_ctx) { set_err("g4o_forward: context exceeds max_ctx"); return -1; }
    const uint32_t d = h->d_model, f = h->d_ff, V = h->vocab_size;
    if (token >= V) {
        if (V < 262144) token %= V;
        else { set_err("Token ID exceeds vocab size"); return -1; }
    }
    /* gbuf/ubuf hold the widest FFN row, and gbuf also the per-layer-input gate [ple_dim]. */
    uint32_t widest = f > h->ple_dim ? f : h->ple_dim;
    for (uint32_t l = 0; l < h->num_layers; ++l)
        if (m->layers[l].ffn > widest) widest = m->layers[l].ffn;
    float* hidden = (float*)malloc(sizeof(float) * d);
    float* norm = (float*)malloc(sizeof(float) * d);
    float* attn = (float*)malloc(sizeof(float) * d);
    float* ffn = (float*)malloc(sizeof(float) * d);
    float* gbuf = (float*)malloc(sizeof(float) * widest);
    float* ubuf = (float*)malloc(sizeof(float) * widest);
    float* wn = (float*)malloc(sizeof(float) * d);

    /* embedding dequant x sqrt(d): src/cpu_reference.cpp:260-291 */
    dequant_int4(m->embed.w + (size_t)token * (d / 8), m->embed.s + (size_t)token * (d / 64),
                 m->embed.b + (size_t)token * (d / 64), 1, d, hidden);
    const float es = sqrtf((float)d);
    for (uint32_t i = 0; i < d; ++i) hidden[i] *= es;

    /* Per-layer inputs, src/runner.cpp:960-1085: the token's row of the per-layer table times
     * sqrt(ple_dim), plus the projection of the scaled embedding with each layer's ple_dim slice
     * RMS-normalised (its hidden^-0.5 factor cancels in that norm and is not applied), both
     * times 2^-0.5. */
    const uint32_t ple = h->ple_dim, ple_rows = h->num_layers * ple;
    float* combined = NULL;
    if (ple) {
        combined = (float*)malloc(sizeof(float) * ple_rows);
        float* tokrow = (float*)malloc(sizeof(float) * ple_rows);
        const uint32_t pt = token % h->ple_vocab;
        dequant_int4(m->ple_table.w + (size_t)pt * (ple_rows / 8), m->ple_table.s + (size_t)pt * (ple_rows / 64),
                     m->ple_table.b + (size_t)pt * (ple_rows / 64), 1, ple_rows, tokrow);
        const float ps = sqrtf((float)ple);
        for (uint32_t i = 0; i < ple_rows; ++i) tokrow[i] *= ps;
        qgemv(&m->ple_model_proj, hidden, combined);
        float* pw = (float*)malloc(sizeof(float) * ple);
        bf16_vec(m->ple_norm, ple, pw);
        for (uint32_t l = 0; l < h->num_layers; ++l) rms_norm_f(combined + (size_t)l * ple, pw, ple, 1e-6f, combined + (size_t)l * ple);
        for (uint32_t i = 0; i < ple_rows; ++i) combined[i] = (combined[i] + tokrow[i]) * 0.70710678118654752f;
        free(pw);
        free(tokrow);
    }

    for (uint32_t l = 0; l < h->num_layers; ++l) {
        layer_t* L = &m->layers[l];
        const uint32_t hd = L->hd, qrows = L->qh * hd, kvrows = L->kvh * hd;
        float* qb = (float*)malloc(sizeof(float) * qrows);
        float* kb = (float*)malloc(sizeof(float) * kvrows);
        float* vb = (float*)calloc(kvrows, sizeof(float));
        float* qn = (float*)malloc(sizeof(float) * hd);
        float* kn = (float*)malloc(sizeof(float) * hd);
        float* head_out = (float*)calloc(qrows, sizeof(float));
        bf16_vec(L->q_norm, hd, qn);
        if (!L->shared) bf16_vec(L->k_norm, hd, kn);

        bf16_vec(L->in_norm, d, wn);
        rms_norm_f(hidden, wn, d, 1e-6f, norm);
        qgemv(&L->q, norm, qb);
        if (!L->shared) qgemv(&L->k, norm, kb);
        if (L->has_v) qgemv(&L->v, norm, vb);

        const float theta = L->is_global ? h->rope_theta_global : h->rope_theta_local;
        const uint32_t rotated = L->is_global ? 64u : hd / 2;
        for (uint32_t hh = 0; hh < L->qh; ++hh) {
            float* qv = qb + (size_t)hh * hd;
            rms_norm_f(qv, qn, hd, 1e-6f, qv);
            rope(qv, hd, rotated, theta, pos);
        }
        if (!L->shared) {
            for (uint32_t hh = 0; hh < L->kvh; ++hh) {
                float* kv = kb + (size_t)hh * hd;
                float* vv = vb + (size_t)hh * hd;
                /* V = unweighted norm of v, or of RAW k on layers without v_proj (:473-477) */
                rms_norm_f(L->has_v ? vv : kv, NULL, hd, 1e-6f, vv);
                rms_norm_f(kv, kn, hd, 1e-6f, kv);
                rope(kv, hd, rotated, theta, pos);
            }
            /* KV cache at reduced precision (:495-498) */
            float* kd = L->kcache + (size_t)pos * kvrows;
            float* vd = L->vcache + (size_t)pos * kvrows;
            for (uint32_t i = 0; i < kvrows; ++i) {
                kd[i] = kv_round(m->kv_mode, kb[i]);
                vd[i] = kv_round(m->kv_mode, vb[i]);
            }
        }
        /* A shared layer attends over its donor's cache, which the donor (an earlier layer of the
         * same type and geometry) has already written for this position (src/runner.cpp:1240-1250). */
        const layer_t* C = &m->layers[L->donor];
        const uint32_t total = pos + 1;
        const uint32_t win = L->is_global ? total : (total < h->sliding_window ? total : h->sliding_window);
        float* scores = (float*)malloc(sizeof(float) * win);
        const uint32_t gqa = L->qh / L->kvh;
        for (uint32_t hh = 0; hh < L->qh; ++hh)
            attend_row(qb + (size_t)hh * hd, C->kcache, C->vcache, L->kvh, hh / gqa, hd,
                       total - win, total, 1.0f, scores, head_out + (size_t)hh * hd);
        free(scores);

        qgemv(&L->o, head_out, attn);
        bf16_vec(L->post_attn_norm, d, wn);
        rms_norm_f(attn, wn, d, 1e-6f, attn);
        for (uint32_t i = 0; i < d; ++i) hidden[i] += attn[i];

        bf16_vec(L->pre_ffn_norm, d, wn);
        rms_norm_f(hidden, wn, d, 1e-6f, norm);
        qgemv(&L->gate, norm, gbuf);
        qgemv(&L->up, norm, ubuf);
        for (uint32_t i = 0; i < L->ffn; ++i) gbuf[i] = g4o_gelu_tanh(gbuf[i]) * ubuf[i];
        qgemv(&L->down, gbuf, ffn);
        bf16_vec(L->post_ffn_norm, d, wn);
        rms_norm_f(ffn, wn, d, 1e-6f, ffn);
        if (!ple) {
            for (uint32_t i = 0; i < d; ++i) hidden[i] = (hidden[i] + ffn[i]) * L->layer_scalar;
        } else {
            /* The per-layer-input block sits between the FFN residual add and layer_scalar
             * (src/runner.cpp:1745-1825): gelu(gate . h) * this layer's slice, projected back to d,
             * normalised, added; the scalar multiplies the sum. */
            for (uint32_t i = 0; i < d; ++i) hidden[i] = hidden[i] + ffn[i];
            qgemv(&L->ple_gate, hidden, gbuf);
            const float* slice = combined + (size_t)l * ple;
            for (uint32_t i = 0; i < ple; ++i) gbuf[i] = g4o_gelu_tanh(gbuf[i]) * slice[i];
            qgemv(&L->ple_proj, gbuf, ffn);
            bf16_vec(L->post_ple_norm, d, wn);
            rms_norm_f(ffn, wn, d, 1e-6f, ffn);
            for (uint32_t i = 0; i < d; ++i) hidden[i] = (hidden[i] + ffn[i]) * L->layer_scalar;
        }

        free(qb); free(kb); free(vb); free(qn); free(kn); free(head_out);
    }
    m->len = pos + 1;

    /* final norm + tied LM head + softcap, src/cpu_reference.cpp:610-665 */
    bf16_vec(m->final_norm, d, wn);
    rms_norm_f(hidden, wn, d, 1e-6f, hidden);
    if (hidden_out) memcpy(hidden_out, hidden, sizeof(float) * d);
    if (logits) {
        qgemv(&m->embed, hidden, logits);
        const float cap = h->final_logit_softcapping;
        if (cap > 0.0f)
            for (uint32_t v = 0; v < V; ++v) logits[v] = cap * tanhf(logits[v] / cap);
    }
    free(hidden); free(norm); free(attn); free(ffn); free(gbuf); free(ubuf); free(wn); free(combined);
    return 0;
}

/* ------------------------------------------------------------------ MTP assistant drafter */

/* G4MtpHeader, include/g4dense/format.hpp:143-180 (packed, 4096 bytes). */
#pragma pack(push, 1)
typedef struct {
    uint32_t magic, version, quant_type, num_layers, backbone_hidden_size, hidden_size, intermediate_size,
        vocab_size, num_q_heads, num_kv_heads, head_dim, global_head_dim, global_kv_heads, sliding_window;
    uint64_t global_layer_mask;
    uint32_t quant_group_size, scale_dtype;
    uint64_t embed_offset, embed_size, pre_proj_offset, pre_proj_size, post_proj_offset, post_proj_size,
        norm_offset, norm_size;
    uint64_t layer_offsets[8], layer_sizes[8];
    uint8_t payload_sha256[32];
    uint8_t reserved[3800];
} g4o_mtp_header;
#pragma pack(pop)

typedef struct {
    uint32_t is_global, qhd;
    const uint16_t *in_norm, *post_attn_norm, *pre_ffn_norm, *post_ffn_norm, *q_norm;
    float layer_scalar;
    qmat q, o, gate, up, down;
} mtp_layer;

struct g4o_mtp {
    g4o_mtp_header h;
    const uint8_t* base;
    size_t size;
    qmat embed, pre, post;
    const uint16_t* norm;
    mtp_layer* layers;
};

/* MtpRunner::load_model + compute_layer_offsets, src/mtp_runner.cpp:92-234, with
 * validate_mtp_header's checks (src/format.cpp:67-130). */
g4o_mtp* g4o_mtp_open(const char* path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { set_err("g4o_mtp_open: cannot open container"); return NULL; }
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(g4o_mtp_header)) {
        close(fd);
        set_err("g4o_mtp_open: container too small for header");
        return NULL;
    }
    void* p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) { set_err("g4o_mtp_open: mmap failed"); return NULL; }
    g4o_mtp* m = (g4o_mtp*)calloc(1, sizeof(g4o_mtp));
    m->base = (const uint8_t*)p;
    m->size = (size_t)st.st_size;
    memcpy(&m->h, p, sizeof(g4o_mtp_header));
    const g4o_mtp_header* h = &m->h;
    int bad = h->magic != 0x47344D54u || h->version != 1 || h->num_layers == 0 || h->num_layers > 8 ||
              !h->backbone_hidden_size || !h->hidden_size || !h->intermediate_size || !h->vocab_size ||
              h->embed_offset % 4096 || h->pre_proj_offset % 4096 || h->post_proj_offset % 4096 ||
              h->norm_offset % 4096;
    for (uint32_t l = 0; !bad && l < h->num_layers; ++l)
        bad = h->layer_offsets[l] % 4096 || !h->layer_sizes[l] || h->layer_offsets[l] + h->layer_sizes[l] > m->size;
    if (bad) {
        set_err("g4o_mtp_open: invalid header");
        munmap(p, m->size);
        free(m);
        return NULL;
    }
    const uint32_t hs = h->hidden_size, bb = h->backbone_hidden_size, I = h->intermediate_size;
    parse_qmat(m->base + h->embed_offset, m->base + h->embed_offset, h->vocab_size, hs, &m->embed);
    parse_qmat(m->base + h->pre_proj_offset, m->base + h->pre_proj_offset, hs, 2 * bb, &m->pre);
    parse_qmat(m->base + h->post_proj_offset, m->base + h->post_proj_offset, bb, hs, &m->post);
    m->norm = (const uint16_t*)(m->base + h->norm_offset);
    m->layers = (mtp_layer*)calloc(h->num_layers, sizeof(mtp_layer));
    for (uint32_t l = 0; l < h->num_layers; ++l) {
        mtp_layer* L = &m->layers[l];
        const uint8_t* lp = m->base + h->layer_offsets[l];
        L->is_global = (uint32_t)((h->global_layer_mask >> l) & 1ull);
        L->qhd = L->is_global ? h->global_head_dim : h->head_dim;
        const uint32_t qd = h->num_q_heads * L->qhd;
        L->in_norm = (const uint16_t*)lp;
        L->post_attn_norm = (const uint16_t*)(lp + hs * 2);
        L->pre_ffn_norm = (const uint16_t*)(lp + hs * 4);
        L->post_ffn_norm = (const uint16_t*)(lp + hs * 6);
        L->q_norm = (const uint16_t*)(lp + hs * 8);
        const uint8_t* sc = lp + hs * 8 + L->qhd * 2;
        L->layer_scalar = g4o_bf16_to_f32(*(const uint16_t*)sc);
        const uint8_t* q = sc + 2;
        q = parse_qmat(lp, q, qd, hs, &L->q);
        q = parse_qmat(lp, q, hs, qd, &L->o);
        q = parse_qmat(lp, q, I, hs, &L->gate);
        q = parse_qmat(lp, q, I, hs, &L->up);
        parse_qmat(lp, q, hs, I, &L->down);
    }
    return m;
}

void g4o_mtp_close(g4o_mtp* m) {
    if (!m) return;
    free(m->layers);
    munmap((void*)m->base, m->size);
    free(m);
}

void g4o_mtp_info(const g4o_mtp* m, uint32_t* o) {
    const g4o_mtp_header* h = &m->h;
    o[0] = h->num_layers; o[1] = h->backbone_hidden_size; o[2] = h->hidden_size; o[3] = h->intermediate_size;
    o[4] = h->vocab_size; o[5] = h->num_q_heads; o[6] = h->num_kv_heads; o[7] = h->head_dim;
    o[8] = h->global_head_dim; o[9] = h->global_kv_heads; o[10] = h->sliding_window;
    o[11] = (uint32_t)h->global_layer_mask;
}

/* MtpRunner::generate_draft_tokens, src/mtp_runner.cpp:263-843. Per step: x = [e(t); h] with
 * e(t) the target's scaled token embedding (src/runner.cpp:2359-2380) and h the target's final
 * normed hidden state (step 0) or the previous step's post-projection; hidden = W_pre x; the
 * layers (q-only attention over the target's KV of its last sliding / last full-attention
 * layer); final norm; post-projection (the next step's h) and the tied LM head (no softcap); the
 * token drawn with sample_token and seed splitmix64(seed + step) (or 1337 + step).
 *
 * Two deliberate differences from the reference, both about positions:
 *   - the reference attends [first, context_length), which includes the pending token's own
 *     position; the target has not processed that token yet, so the slot holds the KV of a
 *     rejected draft or of no token at all. Here the query at position context_length - 1 sees
 *     the keys the target has processed, [max(0, context_length - 1 - window), context_length - 1)
 *     on sliding layers and [0, context_length - 1) on full-attention layers;
 *   - the donor layers, window, RoPE bases and rotated pairs are the target's own (its last
 *     sliding and last full-attention layer; the reference hard-codes 58/59, 1024, 1e4/1e6 and
 *     128/64 pairs, which are the 31B's values).
 * Like the reference, every step uses the same query position and key range. */
int g4o_mtp_draft(const g4o_mtp* mtp, const g4o_model* tgt, const float* target_hidden, uint32_t seed_token,
                  uint32_t context_length, uint32_t k, const g4o_sampling* sp, uint32_t* out_tokens,
                  float* out_logits) {
    const g4o_mtp_header* h = &mtp->h;
    const g4o_header* th = &tgt->h;
    const uint32_t hs = h->hidden_size, bb = h->backbone_hidden_size, I = h->intermediate_size, V = h->vocab_size;
    if (bb != th->d_model || V != th->vocab_size) { set_err("g4o_mtp_draft: drafter does not match the target"); return -1; }
    if (context_length < 2 || context_length - 1 > tgt->len) { set_err("g4o_mtp_draft: bad context length"); return -1; }
    int donor_local = -1, donor_global = -1;
    for (uint32_t l = 0; l < th->num_layers; ++l) {
        if ((th->global_layer_mask >> l) & 1ull) donor_global = (int)l;
        else donor_local = (int)l;
    }
    float* x = (float*)malloc(sizeof(float) * 2 * bb);
    float* hidden = (float*)malloc(sizeof(float) * hs);
    float* norm = (float*)malloc(sizeof(float) * hs);
    float* proj = (float*)malloc(sizeof(float) * hs);
    float* wn = (float*)malloc(sizeof(float) * (hs > 512 ? hs : 512));
    float* gbuf = (float*)malloc(sizeof(float) * I);
    float* ubuf = (float*)malloc(sizeof(float) * I);
    float* post = (float*)malloc(sizeof(float) * bb);
    float* logits = (float*)malloc(sizeof(float) * V);
    const float es = sqrtf((float)bb);
    const uint32_t qpos = context_length - 1, kend = context_length - 1;
    uint32_t tok = seed_token;
    int rc = 0;
    memcpy(post, target_hidden, sizeof(float) * bb);
    for (uint32_t step = 0; step < k; ++step) {
        if (tok >= V) tok %= V;
        dequant_int4(tgt->embed.w + (size_t)tok * (bb / 8), tgt->embed.s + (size_t)tok * (bb / 64),
                     tgt->embed.b + (size_t)tok * (bb / 64), 1, bb, x);
        for (uint32_t i = 0; i < bb; ++i) x[i] *= es;
        memcpy(x + bb, post, sizeof(float) * bb);
        qgemv(&mtp->pre, x, hidden);
        for (uint32_t l = 0; l < h->num_layers; ++l) {
            const mtp_layer* L = &mtp->layers[l];
            const int dl = L->is_global ? donor_global : donor_local;
            if (dl < 0) { set_err("g4o_mtp_draft: target has no donor layer of this kind"); rc = -1; break; }
            const layer_t* D = &tgt->layers[dl];
            const uint32_t qhd = L->qhd, qd = h->num_q_heads * qhd;
            if (D->hd != qhd || D->kvh != (L->is_global ? h->global_kv_heads : h->num_kv_heads)) {
                set_err("g4o_mtp_draft: attention geometry differs from the donor layer");
                rc = -1;
                break;
            }
            float* qb = (float*)malloc(sizeof(float) * qd);
            float* head_out = (float*)calloc(qd, sizeof(float));
            float* qn = (float*)malloc(sizeof(float) * qhd);
            bf16_vec(L->in_norm, hs, wn);
            rms_norm_f(hidden, wn, hs, 1e-6f, norm);
            qgemv(&L->q, norm, qb);
            bf16_vec(L->q_norm, qhd, qn);
            const float theta = L->is_global ? th->rope_theta_global : th->rope_theta_local;
            const uint32_t rotated = L->is_global ? 64u : qhd / 2;
            const uint32_t first = L->is_global ? 0 : (kend > th->sliding_window ? kend - th->sliding_window : 0);
            float* scores = (float*)malloc(sizeof(float) * (kend - first + 1));
            const uint32_t gqa = h->num_q_heads / D->kvh;
            for (uint32_t hh = 0; hh < h->num_q_heads; ++hh) {
                float* qv = qb + (size_t)hh * qhd;
                rms_norm_f(qv, qn, qhd, 1e-6f, qv);
                rope(qv, qhd, rotated, theta, qpos);
                if (kend > first)
                    attend_row(qv, D->kcache, D->vcache, D->kvh, hh / gqa, qhd, first, kend, 1.0f, scores,
                               head_out + (size_t)hh * qhd);
            }
            free(scores);
            qgemv(&L->o, head_out, proj);
            bf16_vec(L->post_attn_norm, hs, wn);
            rms_norm_f(proj, wn, hs, 1e-6f, proj);
            for (uint32_t i = 0; i < hs; ++i) hidden[i] += proj[i];
            bf16_vec(L->pre_ffn_norm, hs, wn);
            rms_norm_f(hidden, wn, hs, 1e-6f, norm);
            qgemv(&L->gate, norm, gbuf);
            qgemv(&L->up, norm, ubuf);
            for (uint32_t i = 0; i < I; ++i) gbuf[i] = g4o_gelu_tanh(gbuf[i]) * ubuf[i];
            qgemv(&L->down, gbuf, proj);
            bf16_vec(L->post_ffn_norm, hs, wn);
            rms_norm_f(proj, wn, hs, 1e-6f, proj);
            for (uint32_t i = 0; i < hs; ++i) hidden[i] = (hidden[i] + proj[i]) * L->layer_scalar;
            free(qb); free(head_out); free(qn);
        }
        if (rc) break;
        bf16_vec(mtp->norm, hs, wn);
        rms_norm_f(hidden, wn, hs, 1e-6f, norm);
        qgemv(&mtp->post, norm, post);
        qgemv(&mtp->embed, norm, logits);
        const uint64_t step_seed = g4o_splitmix64(sp->has_seed ? sp->seed + step : 1337u + step);
        tok = g4o_sample_token(logits, V, sp, step_seed);
        out_tokens[step] = tok;
        if (out_logits) memcpy(out_logits + (size_t)step * V, logits, sizeof(float) * V);
    }
    free(x); free(hidden); free(norm); free(proj); free(wn); free(gbuf); free(ubuf); free(post); free(logits);
    return rc;
}

/* ------------------------------------------------------------------ sampling */

/* src/sampling.cpp:256-261 */
uint64_t g4o_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

/* src/sampling.cpp:263-272 */
uint64_t g4o_seed_for(const g4o_sampling* p, int position) {
    const uint64_t base = p->has_seed ? p->seed + (uint64_t)position
                                      : (0x9E3779B97F4A7C15ULL ^ ((uint64_t)position * 0xD1B54A32D192ED03ULL));
    const uint64_t s = g4o_splitmix64(base);
    return s ? s : 0x9E3779B97F4A7C15ULL;
}

/* validate_sampling, src/sampling.cpp:232-254. Returns 0 or -1. */
int g4o_validate_sampling(const g4o_sampling* p) {
    if (!isfinite(p->temperature) || p->temperature < 0.0f) return -1;
    if (!isfinite(p->top_p) || p->top_p <= 0.0f || p->top_p > 1.0f) return -1;
    if (p->top_k < 0 || p->top_k > 256) return -1;
    if (!isfinite(p->repetition_penalty) || p->repetition_penalty <= 0.0f) return -1;
    if (p->temperature > 0.0f && p->top_p < 1.0f && p->top_k == 0) return -1;
    return 0;
}

/* Greedy argmax, strict '>' so ties keep the lowest index (src/sampling.cpp:297-304). */
uint32_t g4o_argmax(const float* logits, uint32_t vocab) {
    uint32_t best = 0;
    float bv = logits[0];
    for (uint32_t i = 1; i < vocab; ++i)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    return best;
}

static const float* g_sort_logits;
/* by_logit_desc, src/sampling.cpp:328-331: a strict total order. */
static int cmp_desc(const void* a, const void* b) {
    const uint32_t ia = *(const uint32_t*)a, ib = *(const uint32_t*)b;
    const float la = g_sort_logits[ia], lb = g_sort_logits[ib];
    if (la != lb) return la > lb ? -1 : 1;
    return ia < ib ? -1 : (ia > ib);
}

/* xorshift64* uniform, src/sampling.cpp:218-228 */
static float next_uniform(uint64_t* st) {
    uint64_t s = *st;
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    *st = s;
    const uint64_t r = s * 0x2545F4914F6CDD1DULL;
    return (float)((r >> 40) & 0xFFFFFF) / 16777216.0f;
}

/* sample_token, src/sampling.cpp:292-369. The top-`want` shortlist is computed by a full
 * sort under the same strict order, which selects the same elements as nth_element. */
uint32_t g4o_sample_token(const float* logits, uint32_t vocab, const g4o_sampling* p, uint64_t seed) {
    if (p->temperature <= 0.0f) return g4o_argmax(logits, vocab);
    float mx = logits[0];
    for (uint32_t i = 1; i < vocab; ++i) mx = fmaxf(mx, logits[i]);
    double total = 0.0;
    for (uint32_t i = 0; i < vocab; ++i) total += exp((double)logits[i] - mx);
    const size_t want = p->top_k > 0 ? ((size_t)p->top_k < vocab ? (size_t)p->top_k : vocab)
                                     : (256 < vocab ? 256 : vocab);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * vocab);
    for (uint32_t i = 0; i < vocab; ++i) idx[i] = i;
    g_sort_logits = logits;
    qsort(idx, vocab, sizeof(uint32_t), cmp_desc);
    size_t cut = want;
    if (p->top_p < 1.0f) {
        double run = 0.0;
        for (size_t i = 0; i < want; ++i) {
            run += exp((double)logits[idx[i]] - mx) / total;
            if (run >= (double)p->top_p) { cut = i + 1; break; }
        }
    }
    if (p->top_k > 0 && cut > (size_t)p->top_k) cut = (size_t)p->top_k;
    if (cut < 1) cut = 1;
    double* q = (double*)malloc(sizeof(double) * cut);
    double denom = 0.0;
    for (size_t i = 0; i < cut; ++i) {
        q[i] = exp(((double)logits[idx[i]] - mx) / p->temperature);
        denom += q[i];
    }
    uint64_t st = seed;
    const double r = (double)next_uniform(&st) * denom;
    double acc = 0.0;
    uint32_t out = idx[cut - 1];
    for (size_t i = 0; i < cut; ++i) {
        acc += q[i];
        if (acc >= r) { out = idx[i]; break; }
    }
    free(q);
    free(idx);
    return out;
}

/* std::mt19937_64 (the standard's published parameters) */
#define MT_N 312
#define MT_M 156
void g4o_mt64_seed(uint64_t* st, uint64_t seed) {
    st[0] = seed;
    for (int i = 1; i < MT_N; ++i) st[i] = 6364136223846793005ULL * (st[i - 1] ^ (st[i - 1] >> 62)) + (uint64_t)i;
    st[MT_N] = MT_N; /* index */
}

static uint64_t mt64_next(uint64_t* st) {
    const uint64_t UPPER = 0xFFFFFFFF80000000ULL, LOWER = 0x7FFFFFFFULL, A = 0xB5026F5AA96619E9ULL;
    if (st[MT_N] >= MT_N) {
        for (int i = 0; i < MT_N; ++i) {
            const uint64_t y = (st[i] & UPPER) | (st[(i + 1) % MT_N] & LOWER);
            st[i] = st[(i + MT_M) % MT_N] ^ (y >> 1) ^ ((y & 1) ? A : 0);
        }
        st[MT_N] = 0;
    }
    uint64_t z = st[st[MT_N]++];
    z ^= (z >> 29) & 0x5555555555555555ULL;
    z ^= (z << 17) & 0x71D67FFFEDA60000ULL;
    z ^= (z << 37) & 0xFFF7EEE000000000ULL;
    z ^= z >> 43;
    return z;
}

/* uniform_real_distribution<float>(0,1): one 64-bit draw scaled by 2^-64 in float, clamped
 * below 1 (the generate_canonical<float,24> algorithm). */
float g4o_mt64_uniform_float(uint64_t* st) {
    const float sum = (float)mt64_next(st);
    float r = sum / 18446744073709551616.0f;
    if (r >= 1.0f) r = nextafterf(1.0f, 0.0f);
    return r;
}

/* compute_softmax, src/speculator.cpp:14-30 */
static void softmax_t(float* l, uint32_t n, float temp) {
    if (temp <= 0.0f) temp = 1.0f;
    float mx = -1e9f;
    for (uint32_t i = 0; i < n; ++i) {
        l[i] /= temp;
        if (l[i] > mx) mx = l[i];
    }
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        l[i] = expf(l[i] - mx);
        sum += l[i];
    }
    const float inv = 1.0f / (sum > 1e-12f ? sum : 1.0f);
    for (uint32_t i = 0; i < n; ++i) l[i] *= inv;
}

static int is_greedy(const g4o_sampling* p) { return p->temperature <= 0.0f && p->repetition_penalty == 1.0f; }

/* SpeculativeCoordinator::evaluate_verification, src/speculator.cpp:34-153. */
int g4o_evaluate_verification(const uint32_t* drafts, int k_in, const float* target_logits,
                              int n_target, uint32_t vocab, const g4o_sampling* p,
                              uint64_t base_seed, const float* draft_logits,
                              uint32_t* out_tokens, uint32_t* num_accepted) {
    int n_out = 0;
    *num_accepted = 0;
    if (k_in <= 0 || n_target <= 0) return 0;
    const int k = k_in < n_target ? k_in : n_target;
    int accepted = 0;
    float* pt = NULL;
    float* qd = NULL;
    for (int i = 0; i < k; ++i) {
        const uint32_t dt = drafts[i];
        const float* lg = target_logits + (size_t)i * vocab;
        const uint64_t step_seed = g4o_splitmix64(base_seed + (uint64_t)i);
        if (is_greedy(p) || !draft_logits) {
            const uint32_t tt = g4o_sample_token(lg, vocab, p, step_seed);
            if (dt == tt) { out_tokens[n_out++] = dt; ++accepted; }
            else { out_tokens[n_out++] = tt; break; }
            continue;
        }
        if (!pt) { pt = (float*)malloc(sizeof(float) * vocab); qd = (float*)malloc(sizeof(float) * vocab); }
        memcpy(pt, lg, sizeof(float) * vocab);
        softmax_t(pt, vocab, p->temperature);
        memcpy(qd, draft_logits + (size_t)i * vocab, sizeof(float) * vocab);
        softmax_t(qd, vocab, p->temperature);
        const float pv = dt < vocab ? pt[dt] : 0.0f;
        const float qv = dt < vocab ? qd[dt] : 0.0f;
        const float r = qv > 1e-12f ? pv / qv : 1.0f;
        uint64_t mt[MT_N + 1];
        g4o_mt64_seed(mt, step_seed);
        const float u = g4o_mt64_uniform_float(mt);
        if (u <= r) { out_tokens[n_out++] = dt; ++accepted; continue; }
        float sum_diff = 0.0f;
        for (uint32_t v = 0; v < vocab; ++v) {
            const float dd = fmaxf(0.0f, pt[v] - qd[v]);
            qd[v] = dd; /* reuse as diff */
            sum_diff += dd;
        }
        uint32_t corr = 0;
        if (sum_diff > 1e-9f) {
            const float rv = g4o_mt64_uniform_float(mt) * sum_diff;
            float acc = 0.0f;
            for (uint32_t v = 0; v < vocab; ++v) {
                acc += qd[v];
                if (acc >= rv) { corr = v; break; }
            }
        } else {
            corr = g4o_sample_token(lg, vocab, p, step_seed);
        }
        out_tokens[n_out++] = corr;
        break;
    }
    free(pt);
    free(qd);
    if (accepted == k && n_target > k) {
        out_tokens[n_out++] = g4o_sample_token(target_logits + (size_t)k * vocab, vocab, p,
                                               g4o_splitmix64(base_seed + (uint64_t)k));
    }
    *num_accepted = (uint32_t)accepted;
    return n_out;
}

/* ------------------------------------------------------------------ the decode loop */

static uint32_t replay_propose(const uint32_t* stream, int stream_len, int n_prompt, size_t hist_len,
                               double rate, uint64_t seed, uint32_t vocab) {
    const long idx = (long)hist_len - n_prompt;
    const uint32_t truth = (idx >= 0 && idx < stream_len) ? stream[idx] : 0u;
    const uint64_t h = g4o_splitmix64(seed + (uint64_t)hist_len);
    const double u = (double)(h >> 11) * (1.0 / 9007199254740992.0);
    if (u < rate) return (uint32_t)((truth + 1u + (uint32_t)(g4o_splitmix64(h) % (vocab - 1))) % vocab);
    return truth;
}

int g4o_spec_generate(g4o_model* tgt, g4o_model* drf, const uint32_t* prompt, int n_prompt,
                      int max_tokens, int verify_width, const g4o_sampling* sp,
                      double gate_min_accept, int gate_window, int64_t stop_id,
                      const uint32_t* replay_stream, int replay_len, double mismatch_rate,
                      uint64_t mismatch_seed, uint32_t* out_tokens, int* round_info,
                      int max_rounds, int* n_rounds) {
    const uint32_t V = tgt->h.vocab_size;
    size_t cap = (size_t)n_prompt + (size_t)max_tokens + 16;
    uint32_t* hist = (uint32_t*)malloc(sizeof(uint32_t) * cap);
    size_t hn = 0;
    for (int i = 0; i < n_prompt; ++i) {
        uint32_t t = prompt[i];
        if (t >= V) {
            if (V <= 4096) t %= V;
            else { set_err("token id exceeds vocab"); free(hist); return -1; }
        }
        hist[hn++] = t;
    }
    if (hn == 0) { set_err("empty prompt"); free(hist); return -1; }
    g4o_truncate(tgt, 0);
    float* logits = (float*)malloc(sizeof(float) * V);
    for (size_t p = 0; p < hn; ++p)
        if (g4o_forward(tgt, hist[p], (uint32_t)p, logits, NULL)) { free(hist); free(logits); return -1; }
    int emitted = 0, rounds = 0;
#define EMIT(t) (out_tokens[emitted++] = (t))
#define STOP(t) (stop_id >= 0 && (int64_t)(t) == stop_id)
    *n_rounds = 0;
    if (drf && verify_width > 0) {
        g4o_truncate(drf, 0);
        size_t consumed = 0;
        /* The reference caps K at 8 (kGemmMaxBatch); the B200 engine at 16, which BASELINE's k = 8
         * configuration needs. Widths <= 8 behave identically. */
        const uint32_t K = verify_width < 16 ? (uint32_t)verify_width : 16u;
        float* verify = (float*)malloc(sizeof(float) * V * K);
        float* dlog = (float*)malloc(sizeof(float) * V * K);
        uint32_t drafts[16], acc_toks[17];
        uint32_t drafted_total = 0, accepted_total = 0;
        int drafting = 1;
        uint32_t pending = g4o_sample_token(logits, V, sp, g4o_seed_for(sp, (int)(hn - 1)));
        hist[hn++] = pending;
        EMIT(pending);
        if (STOP(pending)) goto done_spec;
        while (emitted < max_tokens) {
            if (!drafting) {
                if (g4o_forward(tgt, pending, (uint32_t)(hn - 1), verify, NULL)) goto fail_spec;
                const uint32_t nx = g4o_sample_token(verify, V, sp, g4o_seed_for(sp, (int)hn));
                hist[hn++] = nx;
                EMIT(nx);
                pending = nx;
                if (STOP(nx)) break;
                continue;
            }
            /* DraftRuntime::generate_draft_tokens, src/draft_runtime.cpp:46-95 */
            if (consumed > hn) consumed = 0;
            g4o_truncate(drf, (uint32_t)consumed);
            while (consumed + 1 < hn) {
                if (g4o_forward(drf, hist[consumed], (uint32_t)consumed, NULL, NULL)) goto fail_spec;
                ++consumed;
            }
            uint32_t cur = hist[hn - 1], pos = (uint32_t)consumed;
            const uint32_t nd = K - 1;
            for (uint32_t step = 0; step < nd; ++step) {
                float* dl = dlog + (size_t)step * V;
                if (g4o_forward(drf, cur, pos, dl, NULL)) goto fail_spec;
                ++pos;
                uint32_t cand;
                if (replay_stream) {
                    cand = replay_propose(replay_stream, replay_len, n_prompt, hn + step, mismatch_rate,
                                          mismatch_seed, V);
                } else {
                    const uint64_t ss = g4o_splitmix64(sp->has_seed ? sp->seed + step : 1337u + step);
                    cand = g4o_sample_token(dl, V, sp, ss);
                }
                drafts[step] = cand;
                cur = cand;
            }
            consumed = hn;
            /* verify pass over [pending, drafts] */
            const uint32_t base = (uint32_t)(hn - 1);
            if (g4o_forward(tgt, pending, base, verify, NULL)) goto fail_spec;
            for (uint32_t i = 0; i < nd; ++i)
                if (g4o_forward(tgt, drafts[i], base + 1 + i, verify + (size_t)(i + 1) * V, NULL)) goto fail_spec;
            uint32_t na = 0;
            const int ne = g4o_evaluate_verification(drafts, (int)nd, verify, (int)K, V, sp,
                                                     g4o_seed_for(sp, (int)hn),
                                                     replay_stream ? NULL : dlog, acc_toks, &na);
            int this_emit = 0, stop = 0;
            for (int i = 0; i < ne; ++i) {
                if (emitted >= max_tokens) { stop = 1; break; }
                hist[hn++] = acc_toks[i];
                EMIT(acc_toks[i]);
                ++this_emit;
                pending = acc_toks[i];
                if (STOP(acc_toks[i])) { stop = 1; break; }
            }
            g4o_truncate(tgt, (uint32_t)(hn - 1));
            consumed = (hn - 1) < g4o_length(drf) ? (hn - 1) : g4o_length(drf);
            if (rounds < max_rounds) {
                round_info[3 * rounds] = (int)nd;
                round_info[3 * rounds + 1] = (int)na;
                round_info[3 * rounds + 2] = this_emit;
            }
            ++rounds;
            drafted_total += nd;
            accepted_total += na;
            if (drafting && gate_window >= 0 && drafted_total >= (uint32_t)gate_window &&
                (double)accepted_total / drafted_total < gate_min_accept)
                drafting = 0;
            if (stop) break;
        }
    done_spec:
        free(verify);
        free(dlog);
        free(hist);
        free(logits);
        *n_rounds = rounds;
        return emitted;
    fail_spec:
        free(verify);
        free(dlog);
        free(hist);
        free(logits);
        return -1;
    }
    /* non-speculative loop, src/runner.cpp:2314-2344 */
    for (int step = 0; step < max_tokens; ++step) {
        const uint32_t nx = g4o_sample_token(logits, V, sp, g4o_seed_for(sp, (int)(hn - 1)));
        hist[hn++] = nx;
        EMIT(nx);
        if (STOP(nx) || emitted >= max_tokens) break;
        if (g4o_forward(tgt, nx, (uint32_t)(hn - 1), logits, NULL)) { free(hist); free(logits); return -1; }
    }
    free(hist);
    free(logits);
    return emitted;
#undef EMIT
#undef STOP
}
