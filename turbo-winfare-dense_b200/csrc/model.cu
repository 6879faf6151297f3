// DeviceModel: residency, layout and the forward pass (see model.h).
//
// Per-layer kernel sequence for M rows (each arrow is one launch, PDL-chained and captured in
// a CUDA graph per M):
//   [qkv GEMM] -> qkv_epi (norms, RoPE, K/V ring) -> attention -> combine (o fragments)
//   -> [o GEMM] -> post_attn (residual, pre-FFN norm) -> [gate|up GEMM] -> geglu
//   -> [down GEMM] -> post_ffn (residual * layer_scalar, next input norm)
// then [LM head GEMM] -> head_chunks (softcap, chunk argmax) -> head_finalize (argmax, greedy
// acceptance). With tensor parallelism the o and down outputs are reduced across ranks with
// one NCCL all-reduce each, and the head's chunk winners with one all-gather.
#include "model.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "common.cuh"
#include "pgemm.h"
#include "shard.h"
#include "synth.h"
#include "vgemm.h"

#ifdef G4B_HAVE_NCCL
#include <nccl.h>
#endif

namespace g4b {

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        std::stringstream ss;
        ss << what << ": " << cudaGetErrorString(e);
        throw std::runtime_error(ss.str());
    }
}

static int round_up(int x, int a) { return (x + a - 1) / a * a; }

DeviceModel::DeviceModel(const ModelOptions& opt) : opt_(opt) {
    if (opt_.tp < 1 || opt_.rank < 0 || opt_.rank >= opt_.tp) throw std::runtime_error("invalid tensor-parallel rank");
#ifndef G4B_HAVE_NCCL
    if (opt_.tp > 1) throw std::runtime_error("tensor parallelism needs the library built with NCCL");
#endif
    if (opt_.stream) {
        stream_ = opt_.stream;
        own_stream_ = false;
    } else {
        cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    cuda_check(cudaHostAlloc((void**)&sp_host_, kParamRing * sizeof(StepParams), cudaHostAllocDefault),
               "cudaHostAlloc");
    cuda_check(cudaHostAlloc((void**)&res_host_, sizeof(HeadResult), cudaHostAllocDefault), "cudaHostAlloc");
}

DeviceModel::~DeviceModel() {
    if (stream_) cudaStreamSynchronize(stream_);
    for (void* p : tp_ipc_open_) cudaIpcCloseMemHandle(p);
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    for (void* p : allocs_) cudaFree(p);
    if (sp_host_) cudaFreeHost(sp_host_);
    if (res_host_) cudaFreeHost(res_host_);
    if (stream_ && own_stream_) cudaStreamDestroy(stream_);
}

void* DeviceModel::dmalloc(size_t bytes) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, std::max<size_t>(bytes, 256)), "cudaMalloc");
    allocs_.push_back(p);
    return p;
}

uint16_t* DeviceModel::upload_u16(const uint16_t* src, size_t n) {
    auto* d = static_cast<uint16_t*>(dmalloc(n * 2));
    cuda_check(cudaMemcpy(d, src, n * 2, cudaMemcpyHostToDevice), "upload");
    return d;
}

void DeviceModel::alloc_qw(QW& q, int N, int K, bool prefill) {
    q.N = N;
    q.K = K;
    q.ktiles = vgemm_ktiles(K);
    q.n_crg = vgemm_n_crg(N);
    q.n_wrg = (N + 63) / 64;
    q.max_slots = vgemm_plan_slots(q.n_crg, q.ktiles);
    q.w = dmalloc(vgemm_weight_bytes(N, K));
    weight_bytes_ += (uint64_t)N * K / 2 + (uint64_t)N * (K / 64) * 4;
    if (prefill && opt_.prefill_tc) {
        q.n_tiles = pgemm_n_tiles(N);
        q.pmax_slots = pgemm_max_slots(q.n_tiles, K / 64, pgemm_grid(q.n_tiles, K / 64));
        q.pw = dmalloc(pgemm_weight_bytes(N, K));
    }
}

// Raw matrix (device pointers, container layout) -> streaming layout (+ prefill layout).
void DeviceModel::upload_qw(QW& q, const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K,
                            bool prefill) {
    alloc_qw(q, N, K, prefill);
    cuda_check(g4b_repack(W, S, B, N, K, q.w, stream_), "repack");
    if (q.pw) cuda_check(pgemm_repack(W, S, B, N, K, q.pw, stream_), "prefill repack");
}

// ----------------------------------------------------------------------------- geometry

namespace {

struct QPtr {
    const uint32_t* w;
    const uint16_t* s;
    const uint16_t* b;
    int rows, cols;
};

// A contiguous row range [r0, r0+n) of a quantized matrix.
struct RowRange {
    const QPtr* m;
    int r0, n;
};

// Host gather of rows (several ranges, concatenated) and a 64-aligned column slice.
void gather_host(const std::vector<RowRange>& ranges, int col0, int Kl, std::vector<uint32_t>& W,
                 std::vector<uint16_t>& S, std::vector<uint16_t>& B) {
    int N = 0;
    for (auto& r : ranges) N += r.n;
    W.resize((size_t)N * (Kl / 8));
    S.resize((size_t)N * (Kl / 64));
    B.resize((size_t)N * (Kl / 64));
    size_t row = 0;
    for (auto& r : ranges) {
        const int K = r.m->cols;
        for (int i = 0; i < r.n; ++i, ++row) {
            const size_t src = (size_t)(r.r0 + i);
            std::memcpy(&W[row * (Kl / 8)], r.m->w + src * (K / 8) + col0 / 8, (Kl / 8) * 4);
            std::memcpy(&S[row * (Kl / 64)], r.m->s + src * (K / 64) + col0 / 64, (Kl / 64) * 2);
            std::memcpy(&B[row * (Kl / 64)], r.m->b + src * (K / 64) + col0 / 64, (Kl / 64) * 2);
        }
    }
}

}  // namespace

// ----------------------------------------------------------------------------- loading

void DeviceModel::load_container(const std::string& path) {
    if (loaded_) throw std::runtime_error("model already loaded");
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) throw G4DenseFormatError("cannot open container " + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(G4DenseHeader)) {
        close(fd);
        throw G4DenseFormatError("container file too small for header");
    }
    const size_t size = (size_t)st.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) throw G4DenseFormatError("mmap failed for " + path);
    struct Unmap {
        void* p;
        size_t n;
        ~Unmap() { munmap(p, n); }
    } unmap{map, size};
    const uint8_t* base = static_cast<const uint8_t*>(map);
    std::memcpy(&h_, base, sizeof(G4DenseHeader));
    validate_header(h_, size);

    const int d = h_.d_model, V = h_.vocab_size;
    // Embedding / tied head block (src/cpu_reference.cpp:260-285, 610-614).
    const uint8_t* emb = base + h_.embed_offset;
    const size_t ew = (size_t)V * (d / 8) * 4, es = (size_t)V * (d / 64) * 2;
    emb_w_ = static_cast<uint32_t*>(dmalloc(ew));
    emb_s_ = static_cast<uint16_t*>(dmalloc(es));
    emb_b_ = static_cast<uint16_t*>(dmalloc(es));
    cuda_check(cudaMemcpy(emb_w_, emb, ew, cudaMemcpyHostToDevice), "upload embed");
    cuda_check(cudaMemcpy(emb_s_, emb + ew, es, cudaMemcpyHostToDevice), "upload embed");
    cuda_check(cudaMemcpy(emb_b_, emb + ew + es, es, cudaMemcpyHostToDevice), "upload embed");
    final_norm_ = upload_u16(reinterpret_cast<const uint16_t*>(emb + ew + 2 * es), d);

    layers_.resize(h_.num_layers);
    for (uint32_t l = 0; l < h_.num_layers; ++l) build_layer_from_host(l, base + h_.layer_offsets[l]);
    finalize_load();
}

void DeviceModel::build_layer_from_host(uint32_t l, const uint8_t* lp) {
    const int d = h_.d_model;
    DevLayer& L = layers_[l];
    L.geo = resolve_layer_geometry(h_, l);
    const int hd = L.geo.head_dim, F = layer_ffn_width(h_, l);
    const Shard sh = make_shard(L.geo, F, opt_.rank, opt_.tp);
    L.hd = hd;
    L.qh = sh.qh_l;
    L.kvh = sh.kvh_l;
    L.F = sh.F_l;
    L.has_v = L.geo.is_global ? 0 : 1;
    L.rotated = L.geo.is_global ? 64 : hd / 2;
    L.theta = L.geo.is_global ? h_.rope_theta_global : h_.rope_theta_local;
    if (L.rotated > hd / 2) throw G4DenseFormatError("global layer head_dim too small for 64 rotary pairs");

    // Norms + layer scalar (src/cpu_reference.cpp:324-356).
    const uint16_t* n = reinterpret_cast<const uint16_t*>(lp);
    L.in_norm = upload_u16(n, d);
    L.pa_norm = upload_u16(n + d, d);
    L.pf_norm = upload_u16(n + 2 * d, d);
    L.pffn_norm = upload_u16(n + 3 * d, d);
    L.q_norm = upload_u16(n + 4 * d, hd);
    L.k_norm = upload_u16(n + 4 * d + hd, hd);
    uint16_t scal;
    std::memcpy(&scal, n + 4 * d + 2 * hd, 2);
    const uint32_t sb = (uint32_t)scal << 16;
    std::memcpy(&L.scalar, &sb, 4);

    // Quant blocks (parse_quant_block, src/cpu_reference.cpp:367-381).
    const uint8_t* p = reinterpret_cast<const uint8_t*>(n + 4 * d + 2 * hd + 1);
    auto parse = [&](int rows, int cols) {
        p += (16u - ((size_t)(p - lp) & 15u)) & 15u;
        QPtr q{reinterpret_cast<const uint32_t*>(p), nullptr, nullptr, rows, cols};
        const size_t wb = (size_t)rows * (cols / 8) * 4, sbytes = (size_t)rows * (cols / 64) * 2;
        q.s = reinterpret_cast<const uint16_t*>(p + wb);
        q.b = reinterpret_cast<const uint16_t*>(p + wb + sbytes);
        p += wb + 2 * sbytes;
        return q;
    };
    const int qrows = L.geo.q_heads * hd, kvrows = L.geo.kv_heads * hd;
    const QPtr Wq = parse(qrows, d), Wk = parse(kvrows, d);
    QPtr Wv{};
    if (L.has_v) Wv = parse(kvrows, d);
    const QPtr Wo = parse(d, qrows), Wg = parse(F, d), Wu = parse(F, d), Wd = parse(d, F);

    std::vector<uint32_t> W;
    std::vector<uint16_t> S, B;
    auto up = [&](QW& q, const std::vector<RowRange>& rr, int col0, int Kl) {
        gather_host(rr, col0, Kl, W, S, B);
        const int N = (int)(S.size() / (Kl / 64));
        uint32_t* dw = static_cast<uint32_t*>(dmalloc(W.size() * 4));
        uint16_t* ds = static_cast<uint16_t*>(dmalloc(S.size() * 2));
        uint16_t* db = static_cast<uint16_t*>(dmalloc(B.size() * 2));
        cuda_check(cudaMemcpy(dw, W.data(), W.size() * 4, cudaMemcpyHostToDevice), "upload");
        cuda_check(cudaMemcpy(ds, S.data(), S.size() * 2, cudaMemcpyHostToDevice), "upload");
        cuda_check(cudaMemcpy(db, B.data(), B.size() * 2, cudaMemcpyHostToDevice), "upload");
        upload_qw(q, dw, ds, db, N, Kl);
        cuda_check(cudaStreamSynchronize(stream_), "repack");
        // the raw staging copies are released right away
        for (void* x : {(void*)dw, (void*)ds, (void*)db}) {
            cudaFree(x);
            allocs_.erase(std::find(allocs_.begin(), allocs_.end(), x));
        }
    };
    std::vector<RowRange> qkv = {{&Wq, sh.q0 * hd, sh.qh_l * hd}, {&Wk, sh.kv0 * hd, sh.kvh_l * hd}};
    if (L.has_v) qkv.push_back({&Wv, sh.kv0 * hd, sh.kvh_l * hd});
    up(L.qkv, qkv, 0, d);
    up(L.o, {{&Wo, 0, d}}, sh.q0 * hd, sh.qh_l * hd);
    up(L.gateup, {{&Wg, sh.f0, sh.F_l}, {&Wu, sh.f0, sh.F_l}}, 0, d);
    up(L.down, {{&Wd, 0, d}}, sh.f0, sh.F_l);
}

void DeviceModel::load_synthetic(const G4DenseHeader& geom, uint64_t seed, bool centered) {
    if (loaded_) throw std::runtime_error("model already loaded");
    h_ = geom;
    h_.magic = G4DenseHeader::kMagic;
    h_.version = G4DenseHeader::kVersion;
    h_.quant_type = 1;
    h_.quant_group_size = 64;
    h_.tied_embeddings = 1;
    const int d = h_.d_model, V = h_.vocab_size;
    if (d % 64 || h_.num_layers == 0 || h_.num_layers > 60) throw G4DenseFormatError("invalid synthetic geometry");
    // Embedding table (replicated) and final norm.
    emb_w_ = static_cast<uint32_t*>(dmalloc((size_t)V * (d / 8) * 4));
    emb_s_ = static_cast<uint16_t*>(dmalloc((size_t)V * (d / 64) * 2));
    emb_b_ = static_cast<uint16_t*>(dmalloc((size_t)V * (d / 64) * 2));
    cuda_check(g4b_synth_qblock(emb_w_, emb_s_, emb_b_, V, d, 0, 0, d, seed, 100000, centered, stream_), "synth");
    final_norm_ = static_cast<uint16_t*>(dmalloc(d * 2));
    cuda_check(g4b_synth_norm(final_norm_, d, seed, 200000, stream_), "synth");

    // Staging for one fused raw matrix at a time.
    size_t max_words = 0;
    layers_.resize(h_.num_layers);
    for (uint32_t l = 0; l < h_.num_layers; ++l) {
        const LayerGeometry g = resolve_layer_geometry(h_, l);
        const Shard sh = make_shard(g, layer_ffn_width(h_, l), opt_.rank, opt_.tp);
        const size_t qkv_rows = (size_t)(sh.qh_l + (g.is_global ? 1 : 2) * sh.kvh_l) * g.head_dim;
        max_words = std::max({max_words, qkv_rows * d / 8, (size_t)d * sh.qh_l * g.head_dim / 8,
                              (size_t)2 * sh.F_l * d / 8, (size_t)d * sh.F_l / 8});
    }
    uint32_t* sw = static_cast<uint32_t*>(dmalloc(max_words * 4));
    uint16_t* ss = static_cast<uint16_t*>(dmalloc(max_words / 8 * 2));
    uint16_t* sbb = static_cast<uint16_t*>(dmalloc(max_words / 8 * 2));

    for (uint32_t l = 0; l < h_.num_layers; ++l) {
        DevLayer& L = layers_[l];
        L.geo = resolve_layer_geometry(h_, l);
        const int hd = L.geo.head_dim, F = layer_ffn_width(h_, l);
        const Shard sh = make_shard(L.geo, F, opt_.rank, opt_.tp);
        L.hd = hd;
        L.qh = sh.qh_l;
        L.kvh = sh.kvh_l;
        L.F = sh.F_l;
        L.has_v = L.geo.is_global ? 0 : 1;
        L.rotated = L.geo.is_global ? 64 : hd / 2;
        L.theta = L.geo.is_global ? h_.rope_theta_global : h_.rope_theta_local;
        // layer_scalar = 1/sqrt(2L) rounded to bf16 (tools/make_synthetic_model.py:143)
        const float sc = 1.0f / std::sqrt(2.0f * (float)h_.num_layers);
        uint32_t u;
        std::memcpy(&u, &sc, 4);
        u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
        std::memcpy(&L.scalar, &u, 4);
        const uint64_t t = (uint64_t)l * 16;
        auto norm = [&](int n, uint64_t id) {
            auto* p = static_cast<uint16_t*>(dmalloc(n * 2));
            cuda_check(g4b_synth_norm(p, n, seed, t + id, stream_), "synth");
            return p;
        };
        L.in_norm = norm(d, 8);
        L.pa_norm = norm(d, 9);
        L.pf_norm = norm(d, 10);
        L.pffn_norm = norm(d, 11);
        L.q_norm = norm(hd, 12);
        L.k_norm = norm(hd, 13);
        // Fused matrices: rows of each sub-matrix are generated from their global indices.
        struct Part {
            uint64_t id;
            int row0_global, rows, Kg;
        };
        auto build = [&](QW& q, const std::vector<Part>& parts, int col0, int Kl) {
            int r = 0;
            for (const Part& pt : parts) {
                cuda_check(g4b_synth_qblock(sw + (size_t)r * (Kl / 8), ss + (size_t)r * (Kl / 64),
                                            sbb + (size_t)r * (Kl / 64), pt.rows, Kl, pt.row0_global, col0, pt.Kg, seed,
                                            t + pt.id, centered, stream_),
                           "synth");
                r += pt.rows;
            }
            upload_qw(q, sw, ss, sbb, r, Kl);
        };
        std::vector<Part> qkv = {{0, sh.q0 * hd, sh.qh_l * hd, d}, {1, sh.kv0 * hd, sh.kvh_l * hd, d}};
        if (L.has_v) qkv.push_back({2, sh.kv0 * hd, sh.kvh_l * hd, d});
        build(L.qkv, qkv, 0, d);
        build(L.o, {{3, 0, d, (int)L.geo.q_heads * hd}}, sh.q0 * hd, sh.qh_l * hd);
        build(L.gateup, {{4, sh.f0, sh.F_l, d}, {5, sh.f0, sh.F_l, d}}, 0, d);
        build(L.down, {{6, 0, d, F}}, sh.f0, sh.F_l);
    }
    cuda_check(cudaStreamSynchronize(stream_), "synthesize");
    for (void* x : {(void*)sw, (void*)ss, (void*)sbb}) {
        cudaFree(x);
        allocs_.erase(std::find(allocs_.begin(), allocs_.end(), x));
    }
    finalize_load();
}

void DeviceModel::finalize_load() {
    const int d = h_.d_model, V = h_.vocab_size;
    if (V % opt_.tp) throw std::runtime_error("vocab must divide by the tensor-parallel size");
    v_local_ = V / opt_.tp;
    v_off_ = opt_.rank * v_local_;
    // The LM head ranks one row of a prefill chunk (its last), so it needs no prefill layout.
    upload_qw(lm_, emb_w_ + (size_t)v_off_ * (d / 8), emb_s_ + (size_t)v_off_ * (d / 64),
              emb_b_ + (size_t)v_off_ * (d / 64), v_local_, d, false);
    // KV rings: sliding layers keep window + max_rows() slots (a batch of rows never overwrites
    // a key an earlier row of the same batch still needs); full-attention layers keep
    // max_context.
    for (auto& L : layers_) {
        if (mtp_) break;  // the MTP drafter attends over its target's rings
        L.cap = L.geo.is_global ? opt_.max_context
                                : std::min<int>(opt_.max_context, (int)h_.sliding_window) + max_rows();
        const size_t n = (size_t)L.cap * L.kvh * L.hd;
        L.k_ring = static_cast<uint16_t*>(dmalloc(n * 2));
        L.v_ring = static_cast<uint16_t*>(dmalloc(n * 2));
        kv_bytes_ += n * 4;
    }
    // Long-context mode (bf16 KV, a context of 8192 or more, or G4DENSE_ATTN_LC=1; =0 turns it
    // off): full-attention layers of head_dim 512 run their verify-batch attention on the
    // tensor cores (attn_lc.cu), which needs TMA maps of their rings and per-split scratch.
    const char* lc_env = std::getenv("G4DENSE_ATTN_LC");
    const bool lc_want = lc_env ? std::atoi(lc_env) != 0 : opt_.max_context >= 8192;
    if (lc_want && opt_.kv_bf16 && !mtp_) {
        size_t pb = 0, mb = 0;
        for (auto& L : layers_) {
            if (!L.geo.is_global || L.hd != 512 || !L.k_ring) continue;
            cuda_check(make_kv_tmap(&L.k_tmap, L.k_ring, L.hd, L.kvh, L.cap), "K ring map");
            cuda_check(make_kv_tmap(&L.v_tmap, L.v_ring, L.hd, L.kvh, L.cap), "V ring map");
            L.lc = true;
            size_t a = 0, b = 0;
            attn_lc_scratch(L.qh, L.kvh, &a, &b);
            pb = std::max(pb, a);
            mb = std::max(mb, b);
        }
        if (pb) {
            lc_part_ = static_cast<float*>(dmalloc(pb));
            lc_ml_ = static_cast<float2*>(dmalloc(mb));
        }
    }
    init_buffers();
    clear_kv();
    cuda_check(cudaStreamSynchronize(stream_), "load");
    loaded_ = true;
}

void DeviceModel::init_buffers() {
    const int d = h_.d_model;
    int max_attn_k = 0, max_F = 0, max_q = 0;
    size_t part = 0, ppart = 0;
    int max_n = d, max_crg = 0, max_tiles = 0;
    auto consider = [&](const QW& q) {
        part = std::max(part, (size_t)q.n_crg * q.max_slots * kMaxM * 256);
        max_crg = std::max(max_crg, q.n_crg);
        if (&q != &lm_) max_n = std::max(max_n, q.N);
        if (q.pw) {
            ppart = std::max(ppart, pgemm_part_floats(q.n_tiles, q.pmax_slots));
            max_tiles = std::max(max_tiles, q.n_tiles);
        }
    };
    for (auto& L : layers_) {
        max_attn_k = std::max(max_attn_k, L.qh * L.hd);
        max_F = std::max(max_F, L.F);
        max_q = std::max(max_q, L.qh * L.hd);
        consider(L.qkv);
        consider(L.o);
        consider(L.gateup);
        consider(L.down);
    }
    consider(lm_);
    if (mtp_) consider(pre_);
    part_floats_ = part;
    const int rows = max_rows();
    for (int i = 0; i < 2; ++i) hres_[i] = static_cast<float*>(dmalloc((size_t)rows * d * 4));
    bf_d_ = dmalloc(bfrag_capacity(round_up(d, 128)));
    bf_attn_ = dmalloc(bfrag_capacity(round_up(max_attn_k, 128)));
    bf_ff_ = dmalloc(bfrag_capacity(round_up(max_F, 128)));
    part_ = static_cast<float*>(dmalloc(part * 4));
    q_buf_ = static_cast<float*>(dmalloc((size_t)rows * max_q * 4));
    y_ = static_cast<float*>(dmalloc((size_t)rows * max_n * 4));
    if (max_tiles) {
        ppart_ = static_cast<float*>(dmalloc(ppart * 4));
        pcnt_ = static_cast<unsigned*>(dmalloc((size_t)max_tiles * sizeof(unsigned)));
        cuda_check(cudaMemset(pcnt_, 0, (size_t)max_tiles * sizeof(unsigned)), "memset");
    }
    cnt_ = static_cast<unsigned*>(dmalloc((size_t)max_crg * sizeof(unsigned)));
    cuda_check(cudaMemset(cnt_, 0, (size_t)max_crg * sizeof(unsigned)), "memset");
    chunk_best_ = static_cast<float2*>(dmalloc((size_t)opt_.tp * kMaxM * g4b_head_chunks(v_local_) * sizeof(float2)));
    logits_ = static_cast<float*>(dmalloc((size_t)kMaxM * v_local_ * 4));
    res_dev_ = static_cast<HeadResult*>(dmalloc(sizeof(HeadResult)));
    sp_dev_ = static_cast<StepParams*>(dmalloc(4 * sizeof(StepParams)));
    chain_dev_ = static_cast<uint32_t*>(dmalloc(64 * 4));
    err_dev_ = static_cast<int*>(dmalloc(sizeof(int)));
    cuda_check(cudaMemsetAsync(err_dev_, 0, sizeof(int), stream_), "memset");
    cuda_check(cudaMemsetAsync(sp_dev_, 0, 4 * sizeof(StepParams), stream_), "memset");
    if (opt_.tp > 1) init_tp_peers();
    if (mtp_) {
        bf_in_ = dmalloc(bfrag_capacity(round_up(pre_.K, 128)));
        post_part_ = static_cast<float*>(dmalloc((size_t)post_.n_crg * post_.max_slots * kMaxM * 256 * 4));
    }
}

void DeviceModel::init_tp_peers() {
#ifdef G4B_HAVE_NCCL
    if (opt_.tp > kMaxTp) throw std::runtime_error("tensor parallelism supports at most 8 ranks");
    const int d = h_.d_model;
    const size_t ybytes = (size_t)2 * max_rows() * d * sizeof(float);
    // Verify rows' push exchange: per parity, one block of {value, epoch} words per source rank.
    const size_t rbytes = (size_t)2 * kMaxTp * kMaxM * d * sizeof(uint2);
    // One cudaMalloc holds both parities, the two flag words and the receive words (IPC maps
    // whole allocations).
    const size_t total = ybytes + 256 + rbytes;
    void* base = dmalloc(total);
    cuda_check(cudaMemset(base, 0, total), "memset");
    tp_buf_ = static_cast<float*>(base);
    tp_flags_ = reinterpret_cast<unsigned*>(static_cast<char*>(base) + ybytes);
    tp_seq_ = static_cast<unsigned*>(dmalloc(sizeof(unsigned)));
    cuda_check(cudaMemset(tp_seq_, 0, sizeof(unsigned)), "memset");
    // Exchange the allocations' IPC handles over the communicator and map every peer's.
    cudaIpcMemHandle_t mine;
    cuda_check(cudaIpcGetMemHandle(&mine, base), "cudaIpcGetMemHandle");
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    char* dh = static_cast<char*>(dmalloc(hb * opt_.tp));
    cuda_check(cudaMemcpy(dh + hb * opt_.rank, &mine, hb, cudaMemcpyHostToDevice), "handle");
    if (ncclAllGather(dh + hb * opt_.rank, dh, hb, ncclChar, (ncclComm_t)opt_.nccl_comm, stream_) != ncclSuccess)
        throw std::runtime_error("ncclAllGather (IPC handles) failed");
    std::vector<cudaIpcMemHandle_t> all(opt_.tp);
    cuda_check(cudaStreamSynchronize(stream_), "sync");
    cuda_check(cudaMemcpy(all.data(), dh, hb * opt_.tp, cudaMemcpyDeviceToHost), "handles");
    for (int r = 0; r < opt_.tp; ++r) {
        void* p = base;
        if (r != opt_.rank) {
            cuda_check(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess),
                       "cudaIpcOpenMemHandle (the ranks' GPUs need peer access)");
            tp_ipc_open_.push_back(p);
        }
        tp_peer_y_[r] = static_cast<float*>(p);
        tp_peer_flags_[r] = reinterpret_cast<unsigned*>(static_cast<char*>(p) + ybytes);
        tp_peer_recv_[r] = reinterpret_cast<uint2*>(static_cast<char*>(p) + ybytes + 256);
    }
#endif
}

TpGather DeviceModel::tp_gather(int step, int parity) const {
    TpGather g{};
    g.n = opt_.tp;
    g.rank = opt_.rank;
    g.step = step;
    g.err = err_dev_;
    if (opt_.tp > 1) {
        const size_t off = (size_t)parity * max_rows() * h_.d_model;
        for (int r = 0; r < opt_.tp; ++r) {
            g.y[r] = tp_peer_y_[r] + off;
            g.flag[r] = tp_peer_flags_[r] + parity;
        }
        g.own_flag = tp_flags_ + parity;
        g.seq = tp_seq_;
        const size_t rrow = (size_t)kMaxM * h_.d_model;
        for (int r = 0; r < opt_.tp; ++r)
            g.push_dst[r] = tp_peer_recv_[r] + ((size_t)parity * kMaxTp + opt_.rank) * rrow;
        g.recv = tp_peer_recv_[opt_.rank] + (size_t)parity * kMaxTp * rrow;
    }
    return g;
}

void DeviceModel::clear_kv() {
    for (auto& L : layers_) {
        if (!L.k_ring) continue;  // the MTP drafter has no rings of its own
        const size_t n = (size_t)L.cap * L.kvh * L.hd * 2;
        cuda_check(cudaMemsetAsync(L.k_ring, 0, n, stream_), "memset kv");
        cuda_check(cudaMemsetAsync(L.v_ring, 0, n, stream_), "memset kv");
    }
}

uint64_t DeviceModel::pass_weight_bytes() const { return weight_bytes_; }

int DeviceModel::kernels_per_pass(int M) const {
    // MTP step: input, pre-projection GEMM, its epilogue; per layer the 9 below; the
    // post-projection and LM head GEMMs, head_chunks and finalize.
    if (mtp_) return 3 + 9 * (int)layers_.size() + 4;
    // embed_norm; per layer 4 GEMMs + qkv_epi + attention + 2 norm/residual epilogues +
    // geglu; LM head GEMM + head_chunks + finalize (NCCL's all-reduce kernels not counted)
    const int per_layer = 9;
    int lc = 0;  // the long-context attention is two kernels (splits, then their combination)
    for (const auto& L : layers_) lc += L.lc && attn_lc_groups(M, L.qh / L.kvh) ? 1 : 0;
    return 1 + per_layer * (int)layers_.size() + lc + 3;
}

double DeviceModel::profile_gemms(int M, int reps, uint64_t* bytes, int* gemm_launches) {
    if (!loaded_) throw std::runtime_error("model not loaded");
    uint64_t b = 0;
    int n = 0;
    auto alg = [&](const QW& q) {
        b += (uint64_t)q.N * q.K / 2 + (uint64_t)q.N * (q.K / 64) * 4 + 4ull * M * q.K + 4ull * M * q.N;
        ++n;
    };
    for (auto& L : layers_) {
        alg(L.qkv);
        alg(L.o);
        alg(L.gateup);
        alg(L.down);
    }
    alg(lm_);
    cudaEvent_t e0, e1;
    cuda_check(cudaEventCreate(&e0), "event");
    cuda_check(cudaEventCreate(&e1), "event");
    cuda_check(cudaEventRecord(e0, stream_), "event");
    for (int r = 0; r < reps; ++r) {
        for (auto& L : layers_) {
            gemm(L.qkv, bf_d_, M, nullptr);
            gemm(L.o, bf_attn_, M, nullptr);
            gemm(L.gateup, bf_d_, M, nullptr);
            gemm(L.down, bf_ff_, M, nullptr);
        }
        gemm(lm_, bf_d_, M, nullptr);
    }
    cuda_check(cudaEventRecord(e1, stream_), "event");
    cuda_check(cudaEventSynchronize(e1), "event");
    float ms = 0.f;
    cuda_check(cudaEventElapsedTime(&ms, e0, e1), "event");
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    launches_ += (uint64_t)n * reps;
    if (bytes) *bytes = b;
    if (gemm_launches) *gemm_launches = n;
    return (double)ms / reps;
}

// ----------------------------------------------------------------------------- forward

PartView DeviceModel::part_view(const QW& q, int M, float* part) const {
    PartView v;
    v.part = part ? part : part_;
    v.max_slots = q.max_slots;
    v.n_crg = q.n_crg;
    v.ktiles = q.ktiles;
    v.grid = vgemm_grid(M, q.n_crg, q.ktiles);
    return v;
}

GemmOut DeviceModel::partials(const QW& q, int M, float* part) const {
    return GemmOut{part_view(q, M, part), nullptr, q.N};
}

float* DeviceModel::tp_out(int parity) const {
    return opt_.tp > 1 ? tp_buf_ + (size_t)parity * max_rows() * h_.d_model : nullptr;
}

void DeviceModel::gemm(const QW& q, const void* bfrag, int M, float* y, float* part) {
    const BFragView v = bfrag_view(const_cast<void*>(bfrag), q.ktiles * 128, M);
    VgemmParams p{};
    p.w = q.w;
    p.bfrag = v.frag;
    p.gsum = v.gsum;
    p.out = part_view(q, M, part);
    p.N = q.N;
    p.M = M;
    p.n_wrg = q.n_wrg;
    p.err = err_dev_;
    p.y = y;  // nullptr: leave the partial slots to the consumer
    p.ldy = q.N;
    p.cnt = cnt_;
    cuda_check(vgemm_launch(p, stream_, opt_.use_pdl), "vgemm");
}

void DeviceModel::pgemm(const QW& q, const void* act, int M, float* y) {
    PgemmParams p{};
    p.w = q.pw;
    p.act = act;
    p.g_layout = q.ktiles * 2;
    p.y = y;
    p.ldy = q.N;
    p.part = ppart_;
    p.cnt = pcnt_;
    p.N = q.N;
    p.K = q.K;
    p.M = M;
    p.n_tiles = q.n_tiles;
    p.max_slots = q.pmax_slots;
    p.err = err_dev_;
    cuda_check(pgemm_launch(p, stream_, opt_.use_pdl), "pgemm");
}

// A prefill chunk of 17..128 rows: the layer kernels of the verify pass with wide-layout
// activations and the tensor-core GEMM (dense outputs), then the LM head on the chunk's last
// row only -- the final norm writes that row alone, in the 1-row fragment layout.
void DeviceModel::enqueue_prefill(int M, bool want_logits) {
    const int d = h_.d_model;
    const bool pdl = opt_.use_pdl;
    StepParams* sp = sp_dev_;
    int cur = 0;
    cuda_check(g4b_embed_norm(sp, emb_w_, emb_s_, emb_b_, h_.vocab_size, d, layers_[0].in_norm, hres_[cur], bf_d_, M,
                              stream_, false),
               "embed_norm");
    for (size_t l = 0; l < layers_.size(); ++l) {
        DevLayer& L = layers_[l];
        pgemm(L.qkv, bf_d_, M, y_);
        QkvEpiArgs qa{};
        qa.qkv = GemmOut{PartView{}, y_, L.qkv.N};
        qa.sp = sp;
        qa.M = M;
        qa.qh = L.qh;
        qa.kvh = L.kvh;
        qa.hd = L.hd;
        qa.has_v = L.has_v;
        qa.rotated = L.rotated;
        qa.theta = L.theta;
        qa.q_norm = L.q_norm;
        qa.k_norm = L.k_norm;
        qa.q_out = q_buf_;
        qa.k_ring = L.k_ring;
        qa.v_ring = L.v_ring;
        qa.cap = L.cap;
        qa.kv_bf16 = opt_.kv_bf16;
        cuda_check(g4b_qkv_epi(qa, stream_, pdl), "qkv_epi");
        AttnArgs aa{};
        aa.q = q_buf_;
        aa.k_ring = L.k_ring;
        aa.v_ring = L.v_ring;
        aa.sp = sp;
        aa.M = M;
        aa.qh = L.qh;
        aa.kvh = L.kvh;
        aa.hd = L.hd;
        aa.cap = L.cap;
        aa.window = L.geo.is_global ? 0 : (int)h_.sliding_window;
        aa.kv_bf16 = opt_.kv_bf16;
        aa.scale = 1.0f;
        if (L.lc && attn_lc_groups(M, L.qh / L.kvh))
            cuda_check(attention_lc(aa, L.k_tmap, L.v_tmap, lc_part_, lc_ml_, err_dev_, bf_attn_, stream_, pdl),
                       "attention_lc");
        else
            cuda_check(g4b_attention(aa, bf_attn_, stream_, pdl), "attention");
        float* yo = opt_.tp > 1 ? tp_out(0) : y_;
        pgemm(L.o, bf_attn_, M, yo);
        cuda_check(g4b_rowepi(GemmOut{PartView{}, yo, d}, tp_gather(2 * (int)l, 0), hres_[cur], hres_[1 - cur],
                              L.pa_norm, 1.0f, L.pf_norm, d, bf_d_, M, stream_, pdl),
                   "post_attn");
        cur = 1 - cur;
        pgemm(L.gateup, bf_d_, M, y_);
        cuda_check(g4b_geglu(GemmOut{PartView{}, y_, L.gateup.N}, L.F, bf_ff_, M, stream_, pdl), "geglu");
        float* yd = opt_.tp > 1 ? tp_out(1) : y_;
        pgemm(L.down, bf_ff_, M, yd);
        const bool last = l + 1 == layers_.size();
        const uint16_t* w_next = last ? final_norm_ : layers_[l + 1].in_norm;
        cuda_check(g4b_rowepi(GemmOut{PartView{}, yd, d}, tp_gather(2 * (int)l + 1, 1), hres_[cur], hres_[1 - cur],
                              L.pffn_norm, L.scalar, w_next, d, bf_d_, M, stream_, pdl, last ? M - 1 : 0,
                              last ? hidden_out_ : nullptr),
                   "post_ffn");
        cur = 1 - cur;
    }
    head(1, want_logits, nullptr, sp);
}

void DeviceModel::enqueue_raw(int M, PassKind kind, bool want_logits, uint32_t* chain_out) {
    if (mtp_) {
        if (M != 1 || (kind != PassKind::MtpFirst && kind != PassKind::MtpNext))
            throw std::runtime_error("the MTP drafter runs one-row MtpFirst / MtpNext steps");
        enqueue_mtp(kind == PassKind::MtpFirst, want_logits, chain_out);
        return;
    }
    if (kind == PassKind::MtpFirst || kind == PassKind::MtpNext) throw std::runtime_error("not an MTP drafter");
    if (M > kMaxM) {
        enqueue_prefill(M, want_logits);
        return;
    }
    const int d = h_.d_model;
    const bool pdl = opt_.use_pdl;
    StepParams* sp = sp_dev_ + (kind == PassKind::DraftStep ? 1 : 0);
    int cur = 0;
    cuda_check(g4b_embed_norm(sp, emb_w_, emb_s_, emb_b_, h_.vocab_size, d, layers_[0].in_norm, hres_[cur], bf_d_, M,
                              stream_, false),
               "embed_norm");
    for (size_t l = 0; l < layers_.size(); ++l) {
        DevLayer& L = layers_[l];
        // Q/K/V
        gemm(L.qkv, bf_d_, M, nullptr);
        QkvEpiArgs qa{};
        qa.qkv = partials(L.qkv, M);
        qa.sp = sp;
        qa.M = M;
        qa.qh = L.qh;
        qa.kvh = L.kvh;
        qa.hd = L.hd;
        qa.has_v = L.has_v;
        qa.rotated = L.rotated;
        qa.theta = L.theta;
        qa.q_norm = L.q_norm;
        qa.k_norm = L.k_norm;
        qa.q_out = q_buf_;
        qa.k_ring = L.k_ring;
        qa.v_ring = L.v_ring;
        qa.cap = L.cap;
        qa.kv_bf16 = opt_.kv_bf16;
        cuda_check(g4b_qkv_epi(qa, stream_, pdl), "qkv_epi");
        // attention
        AttnArgs aa{};
        aa.q = q_buf_;
        aa.k_ring = L.k_ring;
        aa.v_ring = L.v_ring;
        aa.sp = sp;
        aa.M = M;
        aa.qh = L.qh;
        aa.kvh = L.kvh;
        aa.hd = L.hd;
        aa.cap = L.cap;
        aa.window = L.geo.is_global ? 0 : (int)h_.sliding_window;
        aa.kv_bf16 = opt_.kv_bf16;
        aa.scale = 1.0f;
        if (L.lc && attn_lc_groups(M, L.qh / L.kvh))
            cuda_check(attention_lc(aa, L.k_tmap, L.v_tmap, lc_part_, lc_ml_, err_dev_, bf_attn_, stream_, pdl),
                       "attention_lc");
        else
            cuda_check(g4b_attention(aa, bf_attn_, stream_, pdl), "attention");
        // o projection + post-attention norm / residual + pre-FFN norm
        // The o and down GEMMs leave split-K slots. The norm epilogue sums them; under tensor
        // parallelism it first stores this rank's sums into its peer-mapped partial buffer,
        // publishes, and then adds the ranks' partials in rank order over NVLink (TpGather).
        // (Summing in the GEMM's last-arriving CTA instead serialises a long slot list behind
        // one CTA: about 12 us per GEMM at TP = 2.)
        gemm(L.o, bf_attn_, M, nullptr);
        GemmOut oo = partials(L.o, M);
        cuda_check(g4b_rowepi(oo, tp_gather(2 * (int)l, 0), hres_[cur], hres_[1 - cur], L.pa_norm, 1.0f, L.pf_norm, d,
                              bf_d_, M, stream_, pdl),
                   "post_attn");
        cur = 1 - cur;
        // FFN
        gemm(L.gateup, bf_d_, M, nullptr);
        cuda_check(g4b_geglu(partials(L.gateup, M), L.F, bf_ff_, M, stream_, pdl), "geglu");
        gemm(L.down, bf_ff_, M, nullptr);
        GemmOut dn = partials(L.down, M);
        const bool last = l + 1 == layers_.size();
        const uint16_t* w_next = last ? final_norm_ : layers_[l + 1].in_norm;
        cuda_check(g4b_rowepi(dn, tp_gather(2 * (int)l + 1, 1), hres_[cur], hres_[1 - cur], L.pffn_norm, L.scalar,
                              w_next, d, bf_d_, M, stream_, pdl, 0, last ? hidden_out_ : nullptr),
                   "post_ffn");
        cur = 1 - cur;
    }
    head(M, want_logits, chain_out, sp);
}

// LM head over the M rows whose final-norm fragments are in bf_d_ (verify layout), then the
// softcapped chunk argmax and the row argmax / greedy acceptance.
void DeviceModel::head(int M, bool want_logits, uint32_t* chain_out, StepParams* sp, bool advance_pos) {
    const bool pdl = opt_.use_pdl;
    gemm(lm_, bf_d_, M, nullptr);
    const GemmOut lo = partials(lm_, M);
    // Under tensor parallelism each rank ranks its own vocabulary slice; the per-chunk bests
    // (global indices) are all-gathered and every rank finalizes the same argmax.
    const int nch = g4b_head_chunks(v_local_);
    const size_t slice = (size_t)M * nch;
    float2* mine = chunk_best_ + (size_t)opt_.rank * slice;
    cuda_check(g4b_head_chunks_launch(lo, v_local_, M, h_.final_logit_softcapping, want_logits ? logits_ : nullptr,
                                      v_local_, mine, v_off_, stream_, pdl),
               "head_chunks");
#ifdef G4B_HAVE_NCCL
    if (opt_.tp > 1 && ncclAllGather(mine, chunk_best_, slice * 2, ncclFloat, (ncclComm_t)opt_.nccl_comm, stream_) !=
                           ncclSuccess)
        throw std::runtime_error("ncclAllGather (LM head) failed");
#endif
    cuda_check(g4b_head_finalize(chunk_best_, nch, opt_.tp, M, sp, res_dev_, chain_out, opt_.tp > 1 ? tp_seq_ : nullptr,
                                 stream_, pdl, advance_pos),
               "head_finalize");
}

void DeviceModel::logits_to_host(int row0, int rows, float* dst) {
    const size_t VL = (size_t)v_local_;
    if (row0 < 0 || rows < 1 || row0 + rows > kMaxM) throw std::invalid_argument("logits_to_host: rows");
    if (opt_.tp == 1) {
        cuda_check(cudaMemcpyAsync(dst, logits_ + (size_t)row0 * VL, (size_t)rows * VL * 4, cudaMemcpyDeviceToHost,
                                   stream_),
                   "logits");
        d2h_bytes_ += (uint64_t)rows * VL * 4;
        cuda_check(cudaStreamSynchronize(stream_), "logits");
        return;
    }
#ifdef G4B_HAVE_NCCL
    if (!logits_gather_) logits_gather_ = static_cast<float*>(dmalloc((size_t)opt_.tp * kMaxM * VL * 4));
    const size_t n = (size_t)rows * VL;
    if (ncclAllGather(logits_ + (size_t)row0 * VL, logits_gather_, n, ncclFloat, (ncclComm_t)opt_.nccl_comm,
                      stream_) != ncclSuccess)
        throw std::runtime_error("ncclAllGather (logits) failed");
    logits_stage_.resize((size_t)opt_.tp * n);
    cuda_check(cudaMemcpyAsync(logits_stage_.data(), logits_gather_, logits_stage_.size() * 4, cudaMemcpyDeviceToHost,
                               stream_),
               "logits");
    d2h_bytes_ += logits_stage_.size() * 4;
    cuda_check(cudaStreamSynchronize(stream_), "logits");
    // Gathered as [rank][row][vocab slice]; rank r's slice starts at vocabulary id r * VL.
    const size_t V = VL * opt_.tp;
    for (int r = 0; r < opt_.tp; ++r)
        for (int i = 0; i < rows; ++i)
            std::memcpy(dst + (size_t)i * V + (size_t)r * VL, logits_stage_.data() + (size_t)r * n + (size_t)i * VL,
                        VL * 4);
#else
    throw std::runtime_error("logits_to_host: tensor parallelism needs NCCL");
#endif
}

void DeviceModel::bcast_step_tokens(int n) {
    if (opt_.tp == 1 || n <= 0) return;
#ifdef G4B_HAVE_NCCL
    uint32_t* t = sp_dev_[0].tokens + 1;
    if (ncclBroadcast(t, t, (size_t)n, ncclUint32, 0, (ncclComm_t)opt_.nccl_comm, stream_) != ncclSuccess)
        throw std::runtime_error("ncclBroadcast (draft tokens) failed");
#endif
}

void DeviceModel::bcast_host_u32(uint32_t* v, int n) {
    if (opt_.tp == 1 || n <= 0) return;
#ifdef G4B_HAVE_NCCL
    constexpr int kMax = 4 * kPrefillRows;
    if (n > kMax) throw std::invalid_argument("bcast_host_u32: too many words");
    if (!bcast_buf_) bcast_buf_ = static_cast<uint32_t*>(dmalloc(kMax * sizeof(uint32_t)));
    if (opt_.rank == 0) {
        cuda_check(cudaMemcpyAsync(bcast_buf_, v, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), "bcast");
        h2d_bytes_ += (uint64_t)n * 4;
    }
    if (ncclBroadcast(bcast_buf_, bcast_buf_, (size_t)n, ncclUint32, 0, (ncclComm_t)opt_.nccl_comm, stream_) !=
        ncclSuccess)
        throw std::runtime_error("ncclBroadcast (host words) failed");
    if (opt_.rank != 0) {
        cuda_check(cudaMemcpyAsync(v, bcast_buf_, (size_t)n * 4, cudaMemcpyDeviceToHost, stream_), "bcast");
        d2h_bytes_ += (uint64_t)n * 4;
    }
    cuda_check(cudaStreamSynchronize(stream_), "bcast");
#endif
}

void DeviceModel::enqueue(int M, PassKind kind, bool want_logits, uint32_t* chain_out) {
    if (!loaded_) throw std::runtime_error("model not loaded");
    if (M < 1 || M > max_rows())
        throw std::runtime_error("batch width must be 1.." + std::to_string(max_rows()));
    if (opt_.tp > 1 && h_.vocab_size % opt_.tp) throw std::runtime_error("vocab split");
    launches_ += kernels_per_pass(M);
    if (!opt_.use_graphs) {
        enqueue_raw(M, kind, want_logits, chain_out);
        return;
    }
    const auto key = std::make_tuple(M, (int)kind, want_logits, (uintptr_t)chain_out);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
        cudaGraph_t g = nullptr;
        cuda_check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "capture begin");
        try {
            enqueue_raw(M, kind, want_logits, chain_out);
        } catch (...) {
            cudaStreamEndCapture(stream_, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        cuda_check(cudaStreamEndCapture(stream_, &g), "capture end");
        cudaGraphExec_t ge = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        cuda_check(e, "graph instantiate");
        it = graphs_.emplace(key, ge).first;
    }
    cuda_check(cudaGraphLaunch(it->second, stream_), "graph launch");
}

void DeviceModel::push_params(int slot, const StepParams& p, int ntok) {
    // A ring entry is reused only after the stream has drained every earlier copy.
    if (sp_ring_ == kParamRing) {
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        sp_ring_ = 0;
    }
    StepParams& s = sp_host_[sp_ring_++];
    s = p;
    const size_t bytes = offsetof(StepParams, tokens) + (size_t)std::max(1, std::min(ntok, kPrefillRows)) * 4;
    cuda_check(cudaMemcpyAsync(sp_dev_ + slot, &s, bytes, cudaMemcpyHostToDevice, stream_), "params");
    h2d_bytes_ += bytes;
}

void DeviceModel::run_plain(int M, int base_pos, const uint32_t* tokens, bool want_logits) {
    StepParams s;
    std::memset(&s, 0, sizeof(s));
    s.base_pos = base_pos;
    for (int i = 0; i < M; ++i) {
        uint32_t t = tokens[i];
        if (t >= h_.vocab_size) t %= h_.vocab_size;
        s.tokens[i] = t;
    }
    push_params(0, s, std::max(M, kMaxM));
    enqueue(M, PassKind::Plain, want_logits, nullptr);
}

void DeviceModel::rep_reset(const uint32_t* toks, int n) {
    const int V = v_local_;
    if (!rep_count_) {
        rep_count_ = static_cast<uint32_t*>(dmalloc((size_t)V * 4));
        rep_ids_ = static_cast<uint32_t*>(dmalloc((size_t)V * 4));
        rep_stage_ = static_cast<uint32_t*>(dmalloc((size_t)opt_.max_context * 4));
        rep_n_ = static_cast<int*>(dmalloc(sizeof(int)));
    }
    if (n > opt_.max_context) throw std::invalid_argument("repetition history exceeds the context");
    cuda_check(cudaMemsetAsync(rep_count_, 0, (size_t)V * 4, stream_), "memset");
    cuda_check(cudaMemsetAsync(rep_n_, 0, sizeof(int), stream_), "memset");
    cuda_check(cudaMemcpyAsync(rep_stage_, toks, (size_t)n * 4, cudaMemcpyHostToDevice, stream_), "history");
    h2d_bytes_ += (uint64_t)n * 4;
    cuda_check(g4b_rep_append(rep_count_, rep_ids_, rep_n_, rep_stage_, n, V, stream_), "history");
    cuda_check(cudaStreamSynchronize(stream_), "history");  // the pageable source may be reused
}

uint32_t DeviceModel::sample_device(int row, float temperature, float top_p, int top_k, uint64_t seed,
                                    float penalty) {
    if (opt_.tp > 1) throw std::runtime_error("device sampling needs the full vocabulary on one rank");
    if (!sample_work_) {
        sample_work_ = dmalloc(g4b_sample_workspace_bytes());
        sample_out_ = static_cast<uint32_t*>(dmalloc(sizeof(uint32_t)));
    }
    const int V = v_local_;
    const bool pen = penalty != 1.0f;
    if (pen && !rep_count_) throw std::runtime_error("repetition penalty without a history (rep_reset)");
    if (pen) {
        const float cap = h_.final_logit_softcapping;
        cuda_check(g4b_rep_penalty(logits_ + (size_t)row * V, rep_count_, rep_ids_, rep_n_, penalty,
                                   cap > 0.f ? cap * 0.9999f : 0.f, stream_),
                   "repetition penalty");
    }
    cuda_check(g4b_sample_launch(logits_ + (size_t)row * V, V, temperature, top_p, top_k, seed, sample_work_,
                                 sample_out_, stream_),
               "sample");
    launches_ += 2;
    if (pen) {
        cuda_check(g4b_rep_append(rep_count_, rep_ids_, rep_n_, sample_out_, 1, V, stream_), "history");
        launches_ += 2;
    }
    cuda_check(cudaMemcpyAsync(&res_host_->tokens[0], sample_out_, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_),
               "sampled token");
    d2h_bytes_ += sizeof(uint32_t);
    cuda_check(cudaStreamSynchronize(stream_), "sync");
    return res_host_->tokens[0];
}

HeadResult DeviceModel::fetch_result() {
    cuda_check(cudaMemcpyAsync(res_host_, res_dev_, sizeof(HeadResult), cudaMemcpyDeviceToHost, stream_), "result");
    d2h_bytes_ += sizeof(HeadResult);
    cuda_check(cudaStreamSynchronize(stream_), "sync");
    sp_ring_ = 0;  // the stream is drained: the whole parameter ring is free again
    return *res_host_;
}

void DeviceModel::check_device_error() {
    int h = 0;
    cuda_check(cudaMemcpyAsync(&h, err_dev_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "err");
    cuda_check(cudaStreamSynchronize(stream_), "sync");
    if (h) throw std::runtime_error("a kernel's bounded wait gave up (weights or fragments never arrived)");
}

// ----------------------------------------------------------------------------- MTP drafter

void DeviceModel::enable_hidden_out() {
    if (!loaded_) throw std::runtime_error("enable_hidden_out: model not loaded");
    if (mtp_) throw std::runtime_error("enable_hidden_out: not a target model");
    if (hidden_out_) return;
    if (!graphs_.empty()) throw std::runtime_error("enable_hidden_out must precede the first captured pass");
    hidden_out_ = static_cast<float*>(dmalloc((size_t)max_rows() * h_.d_model * 4));
}

// G4DenseHeader fields the shared forward code reads, from the MTP header: the drafter's own
// widths, vocabulary and layer kinds; no softcap on its logits (src/mtp_runner.cpp:773-790).
static G4DenseHeader mtp_as_dense(const G4MtpHeader& m) {
    G4DenseHeader h{};
    h.magic = G4DenseHeader::kMagic;
    h.version = G4DenseHeader::kVersion;
    h.quant_type = 1;
    h.quant_group_size = 64;
    h.num_layers = m.num_layers;
    h.d_model = m.hidden_size;
    h.d_ff = m.intermediate_size;
    h.vocab_size = m.vocab_size;
    h.num_q_heads = m.num_q_heads;
    h.num_kv_heads = m.num_kv_heads;
    h.head_dim = m.head_dim;
    h.global_head_dim = m.global_head_dim;
    h.global_kv_heads = m.global_kv_heads;
    h.sliding_window = m.sliding_window;
    h.global_layer_mask = m.global_layer_mask;
    h.final_logit_softcapping = 0.f;
    h.tied_embeddings = 1;
    return h;
}

void DeviceModel::mtp_attach(DeviceModel& T) {
    if (opt_.tp != 1 || T.opt_.tp != 1) throw std::runtime_error("the MTP drafter runs without tensor parallelism");
    if (!T.loaded_ || T.mtp_) throw std::runtime_error("the MTP drafter needs a loaded target model");
    if (mh_.backbone_hidden_size != T.h_.d_model || mh_.vocab_size != T.h_.vocab_size)
        throw G4DenseFormatError("MTP drafter: backbone width or vocabulary differs from the target's");
    // Donor layers: the target's last sliding and last full-attention layer (the 31B's 58 / 59,
    // src/mtp_runner.cpp:368).
    int donor_local = -1, donor_global = -1;
    for (size_t l = 0; l < T.layers_.size(); ++l) (T.layers_[l].geo.is_global ? donor_global : donor_local) = (int)l;
    for (size_t l = 0; l < layers_.size(); ++l) {
        DevLayer& L = layers_[l];
        const int dl = L.geo.is_global ? donor_global : donor_local;
        if (dl < 0) throw G4DenseFormatError("MTP drafter: the target has no donor layer of this attention kind");
        const DevLayer& D = T.layers_[dl];
        const int want_kvh = L.geo.is_global ? (int)mh_.global_kv_heads : (int)mh_.num_kv_heads;
        if (D.hd != L.hd || D.kvh != want_kvh || L.qh % D.kvh)
            throw G4DenseFormatError("MTP drafter: attention geometry differs from the target's donor layer");
        L.att_k = D.k_ring;
        L.att_v = D.v_ring;
        L.att_cap = D.cap;
        L.att_kvh = D.kvh;
        L.att_window = D.geo.is_global ? 0 : (int)T.h_.sliding_window;
        // Rotation as on the donor: its bases and rotated pairs (the reference hard-codes the
        // 31B's 1e4 / 1e6 and 128 / 64 pairs, src/mtp_runner.cpp:369-372).
        L.theta = D.theta;
        L.rotated = D.rotated;
    }
    donor_ = &T;
    opt_.kv_bf16 = T.opt_.kv_bf16;
}

void DeviceModel::load_mtp(const std::string& path, DeviceModel& target) {
    if (loaded_) throw std::runtime_error("model already loaded");
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) throw G4DenseFormatError("MtpRunner: failed to open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(G4MtpHeader)) {
        close(fd);
        throw G4DenseFormatError("MTP container too small for its header");
    }
    const size_t size = (size_t)st.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) throw G4DenseFormatError("MtpRunner: MapViewOfFile failed for " + path);
    struct Unmap {
        void* p;
        size_t n;
        ~Unmap() { munmap(p, n); }
    } unmap{map, size};
    const uint8_t* base = static_cast<const uint8_t*>(map);
    std::memcpy(&mh_, base, sizeof(G4MtpHeader));
    validate_mtp_header(mh_, size);
    mtp_ = true;
    h_ = mtp_as_dense(mh_);
    const int hs = mh_.hidden_size, bb = mh_.backbone_hidden_size, I = mh_.intermediate_size, V = mh_.vocab_size;
    auto sect = [&](uint64_t off, int rows, int cols) {
        const uint8_t* p = base + off;
        QPtr q{reinterpret_cast<const uint32_t*>(p), nullptr, nullptr, rows, cols};
        const size_t wb = (size_t)rows * (cols / 8) * 4, sb = (size_t)rows * (cols / 64) * 2;
        if (off + wb + 2 * sb > size) throw G4DenseFormatError("MTP section extends beyond the file");
        q.s = reinterpret_cast<const uint16_t*>(p + wb);
        q.b = reinterpret_cast<const uint16_t*>(p + wb + sb);
        return q;
    };
    std::vector<uint32_t> W;
    std::vector<uint16_t> S, B;
    auto up = [&](QW& q, const std::vector<RowRange>& rr, int Kl) {
        gather_host(rr, 0, Kl, W, S, B);
        const int N = (int)(S.size() / (Kl / 64));
        uint32_t* dw = static_cast<uint32_t*>(dmalloc(W.size() * 4));
        uint16_t* ds = static_cast<uint16_t*>(dmalloc(S.size() * 2));
        uint16_t* db = static_cast<uint16_t*>(dmalloc(B.size() * 2));
        cuda_check(cudaMemcpy(dw, W.data(), W.size() * 4, cudaMemcpyHostToDevice), "upload");
        cuda_check(cudaMemcpy(ds, S.data(), S.size() * 2, cudaMemcpyHostToDevice), "upload");
        cuda_check(cudaMemcpy(db, B.data(), B.size() * 2, cudaMemcpyHostToDevice), "upload");
        upload_qw(q, dw, ds, db, N, Kl, false);
        cuda_check(cudaStreamSynchronize(stream_), "repack");
        for (void* x : {(void*)dw, (void*)ds, (void*)db}) {
            cudaFree(x);
            allocs_.erase(std::find(allocs_.begin(), allocs_.end(), x));
        }
    };
    // Tied LM head (the drafter's own [V][hidden] table), projections, final norm
    // (MtpRunner::allocate_gpu_resources, src/mtp_runner.cpp:236-261).
    const QPtr E = sect(mh_.embed_offset, V, hs), Pre = sect(mh_.pre_proj_offset, hs, 2 * bb),
               Post = sect(mh_.post_proj_offset, bb, hs);
    emb_w_ = static_cast<uint32_t*>(dmalloc((size_t)V * (hs / 8) * 4));
    emb_s_ = static_cast<uint16_t*>(dmalloc((size_t)V * (hs / 64) * 2));
    emb_b_ = static_cast<uint16_t*>(dmalloc((size_t)V * (hs / 64) * 2));
    cuda_check(cudaMemcpy(emb_w_, E.w, (size_t)V * (hs / 8) * 4, cudaMemcpyHostToDevice), "upload");
    cuda_check(cudaMemcpy(emb_s_, E.s, (size_t)V * (hs / 64) * 2, cudaMemcpyHostToDevice), "upload");
    cuda_check(cudaMemcpy(emb_b_, E.b, (size_t)V * (hs / 64) * 2, cudaMemcpyHostToDevice), "upload");
    up(pre_, {{&Pre, 0, hs}}, 2 * bb);
    up(post_, {{&Post, 0, bb}}, hs);
    if (mh_.norm_offset + (size_t)hs * 2 > size) throw G4DenseFormatError("MTP norm extends beyond the file");
    final_norm_ = upload_u16(reinterpret_cast<const uint16_t*>(base + mh_.norm_offset), hs);
    // Layers: MtpRunner::compute_layer_offsets (src/mtp_runner.cpp:175-234).
    layers_.resize(mh_.num_layers);
    for (uint32_t l = 0; l < mh_.num_layers; ++l) {
        DevLayer& L = layers_[l];
        const uint8_t* lp = base + mh_.layer_offsets[l];
        L.geo = resolve_layer_geometry(h_, l);
        L.hd = L.geo.head_dim;
        L.qh = mh_.num_q_heads;
        L.kvh = 0;  // q-only: the keys and values are the target's
        L.F = I;
        L.has_v = 0;
        const int qd = L.qh * L.hd;
        const uint16_t* n = reinterpret_cast<const uint16_t*>(lp);
        L.in_norm = upload_u16(n, hs);
        L.pa_norm = upload_u16(n + hs, hs);
        L.pf_norm = upload_u16(n + 2 * hs, hs);
        L.pffn_norm = upload_u16(n + 3 * hs, hs);
        L.q_norm = upload_u16(n + 4 * hs, L.hd);
        uint16_t scal;
        std::memcpy(&scal, n + 4 * hs + L.hd, 2);
        const uint32_t sb = (uint32_t)scal << 16;
        std::memcpy(&L.scalar, &sb, 4);
        const uint8_t* p = reinterpret_cast<const uint8_t*>(n + 4 * hs + L.hd + 1);
        auto parse = [&](int rows, int cols) {
            p += (16u - ((size_t)(p - lp) & 15u)) & 15u;
            QPtr q{reinterpret_cast<const uint32_t*>(p), nullptr, nullptr, rows, cols};
            const size_t wb = (size_t)rows * (cols / 8) * 4, sbytes = (size_t)rows * (cols / 64) * 2;
            q.s = reinterpret_cast<const uint16_t*>(p + wb);
            q.b = reinterpret_cast<const uint16_t*>(p + wb + sbytes);
            p += wb + 2 * sbytes;
            if ((size_t)(p - lp) > mh_.layer_sizes[l]) throw G4DenseFormatError("MTP layer shorter than its matrices");
            return q;
        };
        const QPtr Wq = parse(qd, hs), Wo = parse(hs, qd), Wg = parse(I, hs), Wu = parse(I, hs), Wd = parse(hs, I);
        up(L.qkv, {{&Wq, 0, qd}}, hs);
        up(L.o, {{&Wo, 0, hs}}, qd);
        up(L.gateup, {{&Wg, 0, I}, {&Wu, 0, I}}, hs);
        up(L.down, {{&Wd, 0, hs}}, I);
    }
    mtp_attach(target);
    finalize_load();
}

void DeviceModel::load_mtp_synthetic(const G4MtpHeader& geom, uint64_t seed, bool centered, DeviceModel& target) {
    if (loaded_) throw std::runtime_error("model already loaded");
    mh_ = geom;
    mh_.magic = G4MtpHeader::kMagic;
    mh_.version = G4MtpHeader::kVersion;
    mh_.quant_type = 1;
    mh_.quant_group_size = 64;
    const int hs = mh_.hidden_size, bb = mh_.backbone_hidden_size, I = mh_.intermediate_size, V = mh_.vocab_size;
    if (!mh_.num_layers || mh_.num_layers > G4MtpHeader::kMaxLayers || hs % 64 || bb % 64 || I % 64 || V < 1)
        throw G4DenseFormatError("invalid synthetic MTP geometry");
    mtp_ = true;
    h_ = mtp_as_dense(mh_);
    size_t max_words = (size_t)hs * 2 * bb / 8;
    for (uint32_t l = 0; l < mh_.num_layers; ++l) {
        const LayerGeometry g = resolve_layer_geometry(h_, l);
        max_words = std::max({max_words, (size_t)g.q_heads * g.head_dim * hs / 8, (size_t)2 * I * hs / 8});
    }
    uint32_t* sw = static_cast<uint32_t*>(dmalloc(max_words * 4));
    uint16_t* ss = static_cast<uint16_t*>(dmalloc(max_words / 8 * 2));
    uint16_t* sbb = static_cast<uint16_t*>(dmalloc(max_words / 8 * 2));
    auto build = [&](QW& q, const std::vector<std::pair<uint64_t, int>>& parts, int Kl) {
        int r = 0;
        for (const auto& pt : parts) {
            cuda_check(g4b_synth_qblock(sw + (size_t)r * (Kl / 8), ss + (size_t)r * (Kl / 64), sbb + (size_t)r * (Kl / 64),
                                        pt.second, Kl, 0, 0, Kl, seed, pt.first, centered, stream_),
                       "synth");
            r += pt.second;
        }
        upload_qw(q, sw, ss, sbb, r, Kl, false);
    };
    emb_w_ = static_cast<uint32_t*>(dmalloc((size_t)V * (hs / 8) * 4));
    emb_s_ = static_cast<uint16_t*>(dmalloc((size_t)V * (hs / 64) * 2));
    emb_b_ = static_cast<uint16_t*>(dmalloc((size_t)V * (hs / 64) * 2));
    cuda_check(g4b_synth_qblock(emb_w_, emb_s_, emb_b_, V, hs, 0, 0, hs, seed, 100000, centered, stream_), "synth");
    final_norm_ = static_cast<uint16_t*>(dmalloc(hs * 2));
    cuda_check(g4b_synth_norm(final_norm_, hs, seed, 200000, stream_), "synth");
    build(pre_, {{300000, hs}}, 2 * bb);
    build(post_, {{300001, bb}}, hs);
    layers_.resize(mh_.num_layers);
    for (uint32_t l = 0; l < mh_.num_layers; ++l) {
        DevLayer& L = layers_[l];
        L.geo = resolve_layer_geometry(h_, l);
        L.hd = L.geo.head_dim;
        L.qh = mh_.num_q_heads;
        L.kvh = 0;
        L.F = I;
        L.has_v = 0;
        const float sc = 1.0f / std::sqrt(2.0f * (float)mh_.num_layers);
        uint32_t u;
        std::memcpy(&u, &sc, 4);
        u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
        std::memcpy(&L.scalar, &u, 4);
        const uint64_t t = 400000 + (uint64_t)l * 16;
        auto norm = [&](int n, uint64_t id) {
            auto* p = static_cast<uint16_t*>(dmalloc(n * 2));
            cuda_check(g4b_synth_norm(p, n, seed, t + id, stream_), "synth");
            return p;
        };
        L.in_norm = norm(hs, 8);
        L.pa_norm = norm(hs, 9);
        L.pf_norm = norm(hs, 10);
        L.pffn_norm = norm(hs, 11);
        L.q_norm = norm(L.hd, 12);
        build(L.qkv, {{t + 0, L.qh * L.hd}}, hs);
        build(L.o, {{t + 3, hs}}, L.qh * L.hd);
        build(L.gateup, {{t + 4, I}, {t + 5, I}}, hs);
        build(L.down, {{t + 6, hs}}, I);
    }
    cuda_check(cudaStreamSynchronize(stream_), "synthesize");
    for (void* x : {(void*)sw, (void*)ss, (void*)sbb}) {
        cudaFree(x);
        allocs_.erase(std::find(allocs_.begin(), allocs_.end(), x));
    }
    mtp_attach(target);
    finalize_load();
}

// One MtpRunner::generate_draft_tokens step (src/mtp_runner.cpp:318-843) from StepParams slot 1:
// tokens[0] is the input token, base_pos the last position the target has processed (its
// keys, up to and including base_pos, are what the drafter attends; the query rotates at
// base_pos + 1, the pending token's position) and aux the row of the target's normed hidden
// states a round starts from. With chain_out the drafted token becomes the next step's input
// and is appended to chain_out; the position stays (the reference keeps context_length).
void DeviceModel::enqueue_mtp(bool first, bool want_logits, uint32_t* chain_out) {
    if (!donor_ || !donor_->hidden_out_) throw std::runtime_error("MTP drafter: target hidden states not enabled");
    const int hs = h_.d_model, bb = mh_.backbone_hidden_size;
    const bool pdl = opt_.use_pdl;
    StepParams* sp = sp_dev_ + 1;
    DeviceModel& T = *donor_;
    cuda_check(g4b_mtp_input(sp, T.emb_w_, T.emb_s_, T.emb_b_, T.h_.vocab_size, bb, first ? T.hidden_out_ : nullptr,
                             partials(post_, 1, post_part_), bf_in_, stream_, false),
               "mtp_input");
    gemm(pre_, bf_in_, 1, nullptr);
    int cur = 0;
    const TpGather none = tp_gather(0, 0);
    cuda_check(g4b_rowepi(partials(pre_, 1), none, nullptr, hres_[cur], nullptr, 1.0f, layers_[0].in_norm, hs, bf_d_, 1,
                          stream_, pdl),
               "mtp_pre");
    for (size_t l = 0; l < layers_.size(); ++l) {
        DevLayer& L = layers_[l];
        gemm(L.qkv, bf_d_, 1, nullptr);
        QkvEpiArgs qa{};
        qa.qkv = partials(L.qkv, 1);
        qa.sp = sp;
        qa.M = 1;
        qa.qh = L.qh;
        qa.kvh = 0;
        qa.hd = L.hd;
        qa.rotated = L.rotated;
        qa.theta = L.theta;
        qa.q_norm = L.q_norm;
        qa.q_out = q_buf_;
        qa.kv_bf16 = opt_.kv_bf16;
        qa.pos_offset = 1;
        cuda_check(g4b_qkv_epi(qa, stream_, pdl), "mtp_q_epi");
        AttnArgs aa{};
        aa.q = q_buf_;
        aa.k_ring = L.att_k;
        aa.v_ring = L.att_v;
        aa.sp = sp;
        aa.M = 1;
        aa.qh = L.qh;
        aa.kvh = L.att_kvh;
        aa.hd = L.hd;
        aa.cap = L.att_cap;
        aa.window = L.att_window;
        aa.kv_bf16 = opt_.kv_bf16;
        aa.scale = 1.0f;
        cuda_check(g4b_attention(aa, bf_attn_, stream_, pdl), "mtp_attention");
        gemm(L.o, bf_attn_, 1, nullptr);
        cuda_check(g4b_rowepi(partials(L.o, 1), none, hres_[cur], hres_[1 - cur], L.pa_norm, 1.0f, L.pf_norm, hs, bf_d_,
                              1, stream_, pdl),
                   "mtp_post_attn");
        cur = 1 - cur;
        gemm(L.gateup, bf_d_, 1, nullptr);
        cuda_check(g4b_geglu(partials(L.gateup, 1), L.F, bf_ff_, 1, stream_, pdl), "mtp_geglu");
        gemm(L.down, bf_ff_, 1, nullptr);
        const uint16_t* w_next = (l + 1 < layers_.size()) ? layers_[l + 1].in_norm : final_norm_;
        cuda_check(g4b_rowepi(partials(L.down, 1), none, hres_[cur], hres_[1 - cur], L.pffn_norm, L.scalar, w_next, hs,
                              bf_d_, 1, stream_, pdl),
                   "mtp_post_ffn");
        cur = 1 - cur;
    }
    // Post-projection (the next step's h) into its own slots, then the tied LM head.
    gemm(post_, bf_d_, 1, nullptr, post_part_);
    head(1, want_logits, chain_out, sp, false);
}

}  // namespace g4b
