// One model replica on one GPU: the device-resident counterpart of the
// reference's Model (crates/wasm-chord-runtime/src/transformer/model.rs:19-44).
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "gguf.h"
#include "kernels.h"
#include "sampler.h"

namespace wcb {

struct DevWeight {
  uint8_t* ptr = nullptr;
  int dtype = DT_Q4K;
  uint32_t rows = 0, cols = 0;
  size_t host_off = 0;  // weight streaming: offset in the pinned host copy
};

struct DevLayer {
  DevWeight q, k, v, o, gate, up, down;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
};

struct LoadOptions {
  int device = 0;
  uint32_t max_seq = 0;
  uint32_t kv_half = 0;
  uint32_t max_batch = 1;
  uint32_t flags = 0;
  uint32_t tp_rank = 0;  // tensor parallelism: this process's rank of tp_size
  uint32_t tp_size = 1;
  uint8_t tp_id[128] = {};  // NCCL unique id of the group
  uint32_t wait_ms = 2000;  // bound of every device-side wait on another rank / CTA
};

struct GenParams {
  uint32_t max_tokens = 100;
  float temperature = 0.7f, top_p = 0.9f;
  uint32_t top_k = 40;
  float repetition_penalty = 1.1f;
  uint64_t seed = 42;
  uint32_t eos = 2;
};

class Model {
 public:
  Model(const std::string& path, const LoadOptions& opt);
  ~Model();
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  const ModelConfig& config() const { return cfg_; }
  cudaStream_t stream() const { return stream_; }
  size_t kv_len() const { return kv_len_; }

  // Model::forward (model.rs:832-1192); logits_out (host) may be null
  void forward(const uint32_t* ids, size_t n, size_t position, float* logits_out);
  void clear_kv() { kv_len_ = 0; }
  // Model::generate (model.rs:1322-1415) on token ids
  std::vector<uint32_t> generate(const uint32_t* prompt, size_t n, const GenParams& g);
  // The same loop as a session (the reference's wasmchord_infer / next_token,
  // abi.rs:119-200): start() clears the KV cache, prefills and samples the first
  // token; next() returns up to max_tokens further tokens of the sequence,
  // running decode steps as needed; *finished is set once EOS or max_tokens ends it.
  void start(const uint32_t* prompt, size_t n, const GenParams& g);
  std::vector<uint32_t> next(size_t max_tokens, bool* finished);
  uint64_t session_id() const { return session_; }
  // tensor parallelism: the IPC handle of this rank's receive buffer, and the
  // handles of every rank's (in rank order) to write partial sums into peers
  void tp_ipc_handle(void* out) const;
  void tp_connect(const uint8_t* handles, uint32_t n);
  // tensor parallelism: abandons the group after another rank failed (the
  // caller's watchdog saw it stop): aborts the NCCL communicator, which ends any
  // collective still waiting for that rank; every later call on this model fails.
  // May be called from another thread while a call on this model is blocked.
  void tp_abort();
  // kernels launched by one greedy decode step
  int launches_per_decode_step() const { return launches_per_step_; }
  // generate() for n independent sequences. Greedy decoding with room for
  // several sequences (LoadOptions::max_batch > 1) prefills each sequence into
  // its own KV cache and then runs their decode steps together, up to
  // BATCH_MAX at a time, on the tensor cores; otherwise the sequences run one
  // after the other. Each result is the sequence's generate() result.
  std::vector<std::vector<uint32_t>> generate_batch(const uint32_t* prompts, const size_t* lens, size_t n,
                                                    const GenParams& g);
  // sequences one batched decode step can hold (1: no batched path)
  uint32_t batch_slots() const { return batch_ok_ ? bslots_ : 1; }
  // kernels launched by one batched decode step (0 before the first batched call)
  int launches_per_batch_step() const { return batch_launches_; }

 private:
  // rows [row0, row0 + nrows) and 256-value blocks [blk0, blk0 + nblk) of a
  // [rows][cols] tensor (nrows / nblk 0: all)
  void upload_weight(const GgufFile& f, const std::string& name, uint32_t rows, uint32_t cols, DevWeight& w,
                     bool required_shape_only, uint32_t row0 = 0, uint32_t nrows = 0, uint32_t blk0 = 0,
                     uint32_t nblk = 0, bool to_host = false);
  // weight streaming: copy layer l's weights from the pinned host copy into its
  // device ring slot on the copy stream, after the slot's previous user is done
  void issue_layer_copy(uint32_t l);
  void all_reduce_sum(float* buf, size_t n);  // tensor parallelism: sum over the ranks, in place
  void upload_vector(const GgufFile& f, const std::string& name, uint32_t n, float fill, float*& dst);
  void build_rope(uint32_t len);
  void* dalloc(size_t bytes);
  void set_state(int position, int kv_len, int n_tokens);
  void enqueue_forward(const uint32_t* dev_ids, int T, bool from_hist);
  void enqueue_layers(int T, bool decode = false);
  void enqueue_lm_head(int T, bool gen);
  void gemv(const DevWeight* segs, int nseg, int K, int M, const float* x, int ldx, const float* norm_w, float eps,
            int pro, int epi, float* y, int ldy, const float* resid, int ldr, float* q, int ldq, int layer,
            int token_offset);
  void check(cudaError_t e, const char* what);
  void decode_steps(int steps);
  void capture_decode_graph();
  // greedy prefill of one sequence into the bound KV cache / state, sampling
  // its first token on the device (start()'s greedy path)
  void prefill_greedy(const uint32_t* prompt, size_t n, const GenParams& g);
  // points the per-sequence state (KV cache, StepState, history, penalty
  // counts) at batch slot b; slot 0 is the single-sequence state
  void bind_seq(uint32_t b);
  void enqueue_batch_step(int B);
  // one batched contraction; returns the partial sums of squares it leaves in sq_out
  int batch_gemm(const DevWeight* segs, int nseg, int rows, int K, int B, const float* x, int ldx,
                 const float* norm_w, const float* sq_in, int sq_tiles, float eps, int epi, float* y, int ldy,
                 const float* resid, int ldr, float* sq_out, int layer);
  void build_decode_step();
  bool has_dense_weights() const {  // F32 / F16 2-D weights (the per-op kernels only)
    if (dense_dtype(lm_head_.dtype)) return true;
    for (const DevLayer& L : layers_)
      for (const DevWeight* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
        if (dense_dtype(w->dtype)) return true;
    return false;
  }
  // gen_mode 0: forward of ids_[0]; 1: greedy generate step; 2: logits of a sampled step
  void launch_decode_step_kernel(int gen_mode);
  void enqueue_sampler();  // sampled decoding: penalty, draw and generate()'s bookkeeping

  ModelConfig cfg_;
  LoadOptions opt_;
  // tensor parallelism (Megatron split over tp_ ranks; tp_ == 1: the whole model)
  uint32_t tp_ = 1, rank_ = 0;
  uint32_t hq_ = 0;      // query rows held: hidden / tp
  uint32_t kvd_l_ = 0;   // K (and V) rows held: kv_heads * head_dim / tp
  uint32_t heads_l_ = 0, kv_l_ = 0;
  uint32_t ffn_l_ = 0;   // gate / up rows held and down input columns: ffn / tp
  uint32_t vocab_l_ = 0, vocab_off_ = 0;  // LM-head rows held and the first one's token id
  ncclComm_t comm_ = nullptr;
  std::atomic<bool> tp_failed_{false};  // the group was aborted or a peer wait expired
  void check_group() const;             // throws once the group has failed
  float* part_y_ = nullptr;                 // [t_max][hidden] partial o / down outputs
  unsigned long long* tpkey_ = nullptr;    // argmax key and NaN flag exchanged by the LM head
  // decode steps exchange o / down partial sums by stores into every rank's
  // receive buffer [tp][hidden] of tagged values (CUDA IPC over NVLink)
  unsigned long long* recv_ = nullptr;
  unsigned long long** peers_dev_ = nullptr;  // [tp] device pointers to every rank's recv_
  std::vector<void*> ipc_opened_;
  bool p2p_ = false;
  int peer_phase_ = 0;  // tag phase of the partial sums of the GEMV being enqueued
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  std::vector<void*> allocs_;

  float* emb_ = nullptr;
  float* out_norm_ = nullptr;
  DevWeight lm_head_;
  std::vector<DevLayer> layers_;

  void* kcache_ = nullptr;  // [L][n_kv][max_seq][hd]
  void* vcache_ = nullptr;
  size_t kv_layer_elems_ = 0;
  uint32_t max_seq_ = 0;
  size_t kv_len_ = 0;

  float* rope_cos_ = nullptr;
  float* rope_sin_ = nullptr;
  uint32_t rope_len_ = 0;
  float attn_scale_ = 0.0f;

  int t_max_ = 0;  // tokens per forward launch
  StepState* st_ = nullptr;
  uint32_t* ids_ = nullptr;
  uint32_t* hist_ = nullptr;
  uint32_t hist_cap_ = 0;
  float* x_ = nullptr;
  float* h_ = nullptr;
  float* q_ = nullptr;
  float* att_ = nullptr;
  float* act_ = nullptr;
  float* logits_ = nullptr;
  uint32_t* pen_cnt_ = nullptr;  // occurrences of each token in the sampler history
  float* row_m_ = nullptr;       // per-token RMSNorm divisors for the prefill GEMM
  uint8_t* xprep_ = nullptr;     // the prefill GEMM's activations as fp16 hi / lo tiles
  int gen_mode_ = 0;
  float rep_ = 1.0f;
  int launches_ = 0;
  int launches_per_step_ = 0;
  float* part_ = nullptr;
  int* ticket_ = nullptr;
  int max_splits_ = 0;
  uint32_t* host_ids_ = nullptr;  // pinned staging

  void sync_session_state();

  // session
  uint64_t session_ = 0;
  bool sess_active_ = false;
  bool sess_greedy_ = true;
  bool sess_done_ = true;
  size_t sess_delivered_ = 0;
  size_t sess_steps_left_ = 0;
  GenParams sess_params_;
  std::unique_ptr<Sampler> sess_sampler_;
  std::vector<uint32_t> sess_tokens_;  // host-sampled path: generated ids
  uint32_t sess_last_ = 0;
  StepState sess_state_{};

  // persistent decode step (one cooperative launch per token); with tensor
  // parallelism it runs once the ranks' exchange buffers are connected
  bool mk_ok_ = false;
  bool use_mk() const { return mk_ok_ && (tp_ == 1 || p2p_); }
  // words of the per-op exchange in front of the decode step's region of an exchange buffer
  size_t mk_xofs() const { return size_t(tp_) * cfg_.hidden + 2 * size_t(tp_); }
  MkArgs mk_{};
  size_t mk_smem_ = 0;
  unsigned long long* mk_tagged_ = nullptr;  // tagged activation buffers (one allocation)
  size_t mk_tagged_n_ = 0;
  uint32_t mk_launches_ = 0;

  // weight streaming (LoadOptions::flags bit 4, models larger than the GPU's memory):
  // the layer weights live in pinned host memory and stream through a ring of
  // wslots_ device slots on a copy stream, wslots_ - 1 layers ahead of the compute
  bool wstream_ = false;
  std::vector<uint8_t> wstage_;          // load-time staging of the host copy
  uint8_t* whost_ = nullptr;             // pinned host copy of every layer's weights
  std::vector<size_t> layer_off_, layer_bytes_;
  uint8_t* wring_ = nullptr;             // [wslots_][wslot_bytes_]
  size_t wslot_bytes_ = 0;
  uint32_t wslots_ = 2;
  bool wprimed_ = false;                 // the next forward's first layers are in flight
  cudaStream_t cstream_ = nullptr;
  cudaEvent_t ev_loaded_[2] = {nullptr, nullptr};
  cudaEvent_t ev_free_[2] = {nullptr, nullptr};

 public:
  // weight streaming: host-to-device bytes one forward pass copies (0: weights resident)
  size_t streamed_bytes_per_forward() const {
    size_t t = 0;
    for (size_t b : layer_bytes_) t += b;
    return wstream_ ? t : 0;
  }

 private:
  // batched decode (generate_batch): per-slot state lives in bslots_-long arrays
  // whose slot 0 is the single-sequence state above
  bool batch_ok_ = false;
  uint32_t bslots_ = 1;
  size_t seq_kv_elems_ = 0;     // KV elements of one sequence (all layers)
  void* kc_base_ = nullptr;     // slot 0 caches
  void* vc_base_ = nullptr;
  StepState* st_base_ = nullptr;
  uint32_t* hist_base_ = nullptr;
  uint32_t* pen_base_ = nullptr;
  float* logits_b_ = nullptr;   // [bslots][vocab]
  float* sqx_ = nullptr;        // [tiles x slices][bslots] partial sums of squares of the residual stream x
  float* sqh_ = nullptr;        // the same for h (after attention)
  unsigned long long* tpkeys_b_ = nullptr;  // tensor parallelism: [bslots][2] LM-head keys
  float* apart_ = nullptr;      // attention split partials [bslots][heads][asplits][hd + 2]
  int* aticket_ = nullptr;      // [bslots][kv_heads]
  int asplits_ = 0;
  int batch_launches_ = 0;
  int batch_graph_b_ = 0;
  float batch_graph_rep_ = -1.0f;
  int batch_graph_mode_ = -1;  // the sampler the captured batched step draws with
  float batch_graph_t_ = -1.0f, batch_graph_tp_ = -1.0f;
  int batch_graph_k_ = -1;
  cudaGraphExec_t batch_exec_ = nullptr;
  cudaGraph_t batch_graph_ = nullptr;

  cudaGraphExec_t decode_exec_ = nullptr;
  cudaGraph_t decode_graph_ = nullptr;
  float graph_rep_ = -1.0f;
  int graph_mode_ = -1;                 // sampling mode / parameters the decode graph was captured for
  float graph_t_ = -1.0f, graph_tp_ = -1.0f;
  int graph_k_ = -1;
  // device sampling (sample_dev.cu): mode 1 = top-k / top-p draw on the device
  int sample_mode_ = 0;
  float samp_t_ = 0.0f, samp_tp_ = 0.0f;
  int samp_k_ = 0;
  float* plog_ = nullptr;                 // [vocab] penalised logits
  StdRng* rng_ = nullptr;       // random stream of the bound slot
  StdRng* rng_base_ = nullptr;  // [slot] random streams
  bool sess_host_ = false;                // this session samples on the host
};

}  // namespace wcb
