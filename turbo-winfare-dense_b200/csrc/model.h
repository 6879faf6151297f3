// A fully resident Gemma-4-shaped INT4 G64 model on one GPU (one tensor-parallel shard) and
// its forward pass: ForwardRunner::forward_batch (src/runner.cpp:906-2059) rebuilt as a
// captured CUDA graph of sm_100a kernels per batch width M.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "format.h"
#include "kernels.h"
#include "model_dev.h"

namespace g4b {

struct ModelOptions {
    int max_context = 4096;  // KV capacity of full-attention layers
    int kv_bf16 = 0;         // round K/V through bf16 instead of FP16
    int rank = 0, tp = 1;    // tensor-parallel shard
    void* nccl_comm = nullptr;  // ncclComm_t when tp > 1
    bool use_graphs = true;
    bool use_pdl = true;
    // Keep a second copy of every layer matrix in the prefill GEMM's layout and run prompt
    // chunks of 17..128 rows on the tcgen05 tensor cores (the weights take twice the memory).
    bool prefill_tc = true;
    cudaStream_t stream = nullptr;  // share a caller's stream (target and drafter do)
};

// One INT4 matrix in the vgemm streaming layout (and, for prefill, in the pgemm layout).
struct QW {
    void* w = nullptr;
    int N = 0, K = 0, ktiles = 0, n_crg = 0, n_wrg = 0, max_slots = 0;
    void* pw = nullptr;  // prefill-GEMM layout (nullptr: no tensor-core prefill for this matrix)
    int n_tiles = 0, pmax_slots = 0;
};

struct DevLayer {
    LayerGeometry geo{};
    int qh = 0, kvh = 0, hd = 0;  // local heads
    int has_v = 0, rotated = 0;
    float theta = 0.f, scalar = 1.f;
    int F = 0;                    // local FFN width
    QW qkv, o, gateup, down;
    uint16_t *in_norm = nullptr, *pa_norm = nullptr, *pf_norm = nullptr, *pffn_norm = nullptr;
    uint16_t *q_norm = nullptr, *k_norm = nullptr;
    uint16_t *k_ring = nullptr, *v_ring = nullptr;
    int cap = 0;
    // Long-context mode: TMA maps of the rings for the tensor-core attention (attn_lc.cu).
    bool lc = false;
    KvTmap k_tmap{}, v_tmap{};
    // MTP drafter layers attend over a donor layer of the target instead of their own ring.
    const uint16_t *att_k = nullptr, *att_v = nullptr;
    int att_cap = 0, att_kvh = 0, att_window = 0;
};

// Rows one pass processes at most (verify width, prefill chunk).
constexpr int kBatchRows = 16;

enum class PassKind { Plain = 0, DraftStep = 1, MtpFirst = 2, MtpNext = 3 };

class DeviceModel {
   public:
    explicit DeviceModel(const ModelOptions& opt);
    ~DeviceModel();
    DeviceModel(const DeviceModel&) = delete;
    DeviceModel& operator=(const DeviceModel&) = delete;

    // Reads a .g4dense v3 container (validated like src/format.cpp) and uploads this rank's
    // shard.
    void load_container(const std::string& path);
    // Generates weights with the container's value distributions directly on the device
    // for the geometry in `geom` (header fields only; offsets are ignored).
    void load_synthetic(const G4DenseHeader& geom, uint64_t seed, bool centered);
    // The MTP "assistant" drafter (src/mtp_runner.cpp) as a model of this class: a .g4mtp
    // container (validated like src/format.cpp:67-130), or synthetic weights of that geometry.
    // Its attention reads `target`'s KV rings (the target's last sliding and last full-attention
    // layers) and its input the target's embedding table and final normed hidden states, so the
    // target must outlive it, run tensor-parallel size 1, and have enable_hidden_out() set.
    void load_mtp(const std::string& path, DeviceModel& target);
    void load_mtp_synthetic(const G4MtpHeader& geom, uint64_t seed, bool centered, DeviceModel& target);
    bool is_mtp() const { return mtp_; }
    const G4MtpHeader& mtp_header() const { return mh_; }
    // Makes every pass also write its final normed hidden rows in fp32 ([rows][d_model]; a prefill
    // chunk's last row as row 0), the MTP drafter's input. Call before the first pass.
    void enable_hidden_out();

    const G4DenseHeader& header() const { return h_; }
    int vocab_local() const { return v_local_; }
    int max_context() const { return opt_.max_context; }
    uint64_t weight_bytes() const { return weight_bytes_; }
    uint64_t kv_bytes() const { return kv_bytes_; }
    cudaStream_t stream() const { return stream_; }
    const ModelOptions& options() const { return opt_; }

    // Device step-parameter slots: 0 = plain passes, 1 = drafter chaining.
    StepParams* step_params(int slot) { return sp_dev_ + slot; }
    HeadResult* result_dev() { return res_dev_; }
    float* logits_dev() { return logits_; }  // [16][vocab_local] when a pass asked for them
    // Copies `rows` full-vocabulary logits rows from row `row0` of the last pass that asked for
    // logits into host `dst` ([rows][vocab]) and synchronizes the stream. Under tensor
    // parallelism every rank's vocabulary slice is all-gathered first (every rank must call it,
    // in the same order) and the slices are placed in rank order.
    void logits_to_host(int row0, int rows, float* dst);
    // Tensor parallelism with the drafter on rank 0 only. bcast_step_tokens: on the model's
    // stream, rank 0's StepParams slot-0 tokens [1, 1 + n) (the drafts its drafter chained there)
    // are broadcast into every rank's slot 0, ahead of the verify pass that reads them.
    // bcast_host_u32: rank 0's host words `v[0..n)` replace every rank's (synchronizes). Every
    // rank must call them, in the same order; at tp = 1 they do nothing.
    void bcast_step_tokens(int n);
    void bcast_host_u32(uint32_t* v, int n);
    uint32_t* chain_dev() { return chain_dev_; }

    // Enqueues one pass of M rows on the model's stream (graph-replayed when enabled): 1..16
    // rows run the verify path, 17..max_rows() (prefill chunks) the tensor-core path, which
    // ranks only the last row (its result and logits are row 0). The caller has already
    // written the StepParams slot used by `kind`.
    void enqueue(int M, PassKind kind, bool want_logits, uint32_t* chain_out);
    // Rows one pass may hold, and the result/logits row that holds a pass's last row.
    int max_rows() const { return opt_.prefill_tc ? kPrefillRows : kMaxM; }
    static int result_row(int M) { return M > kMaxM ? 0 : M - 1; }
    // Stages `p` in a pinned ring and enqueues the copy of its first `ntok` tokens (and the
    // scalar fields) into StepParams slot `slot`.
    void push_params(int slot, const StepParams& p, int ntok = kMaxM);
    // Host helper: write StepParams slot 0 (base_pos, tokens) and enqueue a plain pass.
    void run_plain(int M, int base_pos, const uint32_t* tokens, bool want_logits);
    // Copies the result struct to host (synchronizes the stream).
    HeadResult fetch_result();
    // Draws a token on the device from logits row `row` of the last pass that asked for logits
    // (sample_token, src/sampling.cpp:92-169, with the given seed) and returns it (synchronizes
    // the stream; 4 bytes come back instead of the logits row).
    // With penalty != 1 the row is first penalised for the history set by rep_reset and the
    // draws since (apply_repetition_penalty, src/sampling.cpp:74-90), and the drawn token joins it.
    uint32_t sample_device(int row, float temperature, float top_p, int top_k, uint64_t seed, float penalty = 1.0f);
    // Sets the device-side repetition history to `toks` (the prompt).
    void rep_reset(const uint32_t* toks, int n);
    void check_device_error();  // throws if a kernel's bounded wait gave up
    void clear_kv();

    // Timing hook: total verify-GEMM algorithmic weight bytes of one pass.
    uint64_t pass_weight_bytes() const;
    // Kernel launches of one pass of M rows, and the running count of launches enqueued.
    int kernels_per_pass(int M) const;
    uint64_t launches() const { return launches_; }
    // Times every verify GEMM of one M-row pass (PDL-chained, `reps` times back to back) with
    // CUDA events on the model's stream. Returns milliseconds per pass; *bytes receives the
    // algorithmic bytes of one pass's GEMMs (packed weights + fp32 activations + outputs).
    double profile_gemms(int M, int reps, uint64_t* bytes, int* gemm_launches);
    // Host<->device bytes moved by the per-pass parameter and result copies so far.
    uint64_t h2d_bytes() const { return h2d_bytes_; }
    uint64_t d2h_bytes() const { return d2h_bytes_; }

   private:
    void init_buffers();
    void init_tp_peers();  // tensor parallelism: peer-mapped partial buffers and flags
    TpGather tp_gather(int step, int parity) const;
    void build_layer_from_host(uint32_t l, const uint8_t* layer_ptr);
    void enqueue_raw(int M, PassKind kind, bool want_logits, uint32_t* chain_out);
    void enqueue_mtp(bool first, bool want_logits, uint32_t* chain_out);
    void mtp_attach(DeviceModel& target);  // donor rings, geometry checks, buffers
    // One verify GEMM; y == nullptr leaves split-K partials for the consumer (partials()).
    void gemm(const QW& q, const void* bfrag, int M, float* y, float* part = nullptr);
    // One prefill GEMM (17..128 rows, wide-layout activations) into the dense y[M][q.N].
    void pgemm(const QW& q, const void* act, int M, float* y);
    void enqueue_prefill(int M, bool want_logits);
    void head(int M, bool want_logits, uint32_t* chain_out, StepParams* sp, bool advance_pos = true);
    PartView part_view(const QW& q, int M, float* part = nullptr) const;
    GemmOut partials(const QW& q, int M, float* part = nullptr) const;
    float* tp_out(int parity) const;  // under TP: this rank's partial buffer of that parity, else nullptr
    void upload_qw(QW& q, const uint32_t* W, const uint16_t* S, const uint16_t* B, int N, int K,
                   bool prefill = true);
    void alloc_qw(QW& q, int N, int K, bool prefill);
    uint16_t* upload_u16(const uint16_t* src, size_t n);
    void* dmalloc(size_t bytes);
    void finalize_load();

    ModelOptions opt_;
    G4DenseHeader h_{};
    cudaStream_t stream_ = nullptr;
    std::vector<void*> allocs_;
    std::vector<DevLayer> layers_;
    QW lm_;
    // MTP drafter mode: pre-/post-projections, the target whose rings and embedding it reads,
    // the post-projection's own split-K slots (they outlive the LM head's), its input fragments.
    bool mtp_ = false;
    G4MtpHeader mh_{};
    DeviceModel* donor_ = nullptr;
    QW pre_, post_;
    float* post_part_ = nullptr;
    void* bf_in_ = nullptr;
    float* hidden_out_ = nullptr;  // final normed hidden rows (enable_hidden_out)
    int v_local_ = 0, v_off_ = 0;
    uint32_t* emb_w_ = nullptr;
    uint16_t *emb_s_ = nullptr, *emb_b_ = nullptr, *final_norm_ = nullptr;
    // work buffers
    float* hres_[2] = {nullptr, nullptr};
    void* bf_d_ = nullptr;     // B fragments with K = d_model
    void* bf_attn_ = nullptr;  // K = local q_heads * head_dim (max over layers)
    float* lc_part_ = nullptr;   // long-context attention: per-split partial outputs
    float2* lc_ml_ = nullptr;    //   and {max, sum} per row
    void* bf_ff_ = nullptr;    // K = local FFN width
    float* part_ = nullptr;
    size_t part_floats_ = 0;
    float* q_buf_ = nullptr;
    float* y_ = nullptr;       // dense GEMM output [16][max N]
    // tensor parallelism: this rank's [2 parities][16][d] partials + [2] flags (IPC-exported),
    // the peers' mappings, and the pass counter that makes every step's epoch distinct
    float* tp_buf_ = nullptr;
    unsigned* tp_flags_ = nullptr;
    unsigned* tp_seq_ = nullptr;
    uint2* tp_peer_recv_[kMaxTp] = {};  // each rank's receive words [2][tp][16][d] {value, epoch} (peer-mapped)
    float* tp_peer_y_[kMaxTp] = {};
    unsigned* tp_peer_flags_[kMaxTp] = {};
    std::vector<void*> tp_ipc_open_;
    unsigned* cnt_ = nullptr;  // split-K arrival counters of the GEMM running on stream_
    float* ppart_ = nullptr;   // prefill GEMM split-K slots
    unsigned* pcnt_ = nullptr; // prefill GEMM tile arrival counters
    float2* chunk_best_ = nullptr;
    float* logits_ = nullptr;
    float* logits_gather_ = nullptr;  // [tp][16][vocab_local]: all-gathered logits rows (tp > 1)
    uint32_t* bcast_buf_ = nullptr;   // device staging of bcast_host_u32
    std::vector<float> logits_stage_;
    void* sample_work_ = nullptr;      // device sampler workspace (allocated on first use)
    uint32_t* sample_out_ = nullptr;   // device: the sampled token
    uint32_t *rep_count_ = nullptr, *rep_ids_ = nullptr, *rep_stage_ = nullptr;  // repetition history
    int* rep_n_ = nullptr;
    HeadResult* res_dev_ = nullptr;
    StepParams* sp_dev_ = nullptr;
    uint32_t* chain_dev_ = nullptr;
    int* err_dev_ = nullptr;
    uint64_t weight_bytes_ = 0, kv_bytes_ = 0;
    bool loaded_ = false;
    // staging for raw (container-layout) matrices before the repack
    uint32_t* stage_w_ = nullptr;
    uint16_t *stage_s_ = nullptr, *stage_b_ = nullptr;
    size_t stage_words_ = 0;
    std::map<std::tuple<int, int, bool, uintptr_t>, cudaGraphExec_t> graphs_;
    bool pdl_in_graphs_ = true;
    StepParams* sp_host_ = nullptr;  // pinned ring of kParamRing entries
    int sp_ring_ = 0;
    static constexpr int kParamRing = 4096;  // no host stall in a 30k-token prefill
    HeadResult* res_host_ = nullptr; // pinned
    bool own_stream_ = true;
    uint64_t launches_ = 0, h2d_bytes_ = 0, d2h_bytes_ = 0;
};

// cudaError_t -> exception with context.
void cuda_check(cudaError_t e, const char* what);

}  // namespace g4b
