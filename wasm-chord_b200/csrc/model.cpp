#include "model.h"

#include "nccl_rt.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

namespace wcb {

namespace {

constexpr int T_MAX = 2048;       // tokens per forward launch (longer prompts are split, same results)
constexpr int DECODE_CHUNK = 32;  // keys per attention split in decode steps
constexpr int BATCH_CHUNK = 256;  // keys per attention split in batched decode steps

float f16_to_f32_host(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, mant = h & 0x3FF, out;
  if (exp == 0) {
    if (mant == 0) {
      out = sign;
    } else {
      int e = -1;
      do { e++; mant <<= 1; } while (!(mant & 0x400));
      out = sign | (uint32_t(127 - 15 - e) << 23) | ((mant & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (mant << 13);
  } else {
    out = sign | ((exp + 112) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

uint32_t cuda_code(cudaError_t e) { return e == cudaErrorMemoryAllocation ? E_OOM : E_BACKEND; }

}  // namespace

void Model::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw WcbError(cuda_code(e), std::string("Backend error: ") + what + ": " + cudaGetErrorString(e));
}

void* Model::dalloc(size_t bytes) {
  void* p = nullptr;
  check(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc");
  allocs_.push_back(p);
  return p;
}

Model::Model(const std::string& path, const LoadOptions& opt) : opt_(opt), device_(opt.device) {
  GgufFile f(path);
  cfg_ = f.config();
  const ModelConfig& c = cfg_;
  if (c.heads == 0 || c.kv_heads == 0 || c.hidden % c.heads || c.heads % c.kv_heads)
    throw WcbError(E_INVALID, "Invalid tensor shape: heads / kv_heads / hidden are inconsistent");
  const uint32_t hd = c.head_dim();
  if (hd != 64 && hd != 128) throw WcbError(E_BACKEND, "Backend error: head_dim must be 64 or 128");
  if (c.hidden % 256 || c.ffn % 256)
    throw WcbError(E_BACKEND, "Backend error: hidden and intermediate sizes must be multiples of 256");
  if (c.heads / c.kv_heads > 16) throw WcbError(E_BACKEND, "Backend error: more than 16 query heads per KV head");
  if (c.vocab % 4) throw WcbError(E_BACKEND, "Backend error: vocab size must be a multiple of 4");
  max_seq_ = opt.max_seq ? opt.max_seq : c.max_seq;
  if (max_seq_ == 0) throw WcbError(E_INVALID, "Invalid tensor shape: context length 0");
  // the one tensor the reference requires (model.rs:432-446), checked before any device work
  if (!f.find("token_embd.weight") && !f.find("model.embed_tokens.weight") && !f.find("embed_tokens.weight"))
    throw WcbError(E_PARSE, "Parse error: Missing token embeddings");

  tp_ = std::max<uint32_t>(opt.tp_size, 1);
  rank_ = opt.tp_rank;
  if (tp_ > 1) {
    // Megatron split: heads and FFN rows column-parallel, o / down row-parallel
    // (their input columns split), LM head split by vocabulary
    if (c.heads % tp_ || c.kv_heads % tp_ || c.hidden % (QK_K * tp_) || c.ffn % (QK_K * tp_) ||
        c.vocab % (4 * tp_) || (c.ffn / tp_) % 4)
      throw WcbError(E_BACKEND, "Backend error: the model's heads, hidden, intermediate and vocab sizes do not "
                                "split over " + std::to_string(tp_) + " tensor-parallel ranks");
  }
  hq_ = c.hidden / tp_;
  kvd_l_ = c.kv_heads * hd / tp_;
  heads_l_ = c.heads / tp_;
  kv_l_ = c.kv_heads / tp_;
  ffn_l_ = c.ffn / tp_;
  vocab_l_ = c.vocab / tp_;
  vocab_off_ = rank_ * vocab_l_;

  check(cudaSetDevice(device_), "cudaSetDevice");
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  if (tp_ > 1) {
    ncclUniqueId id;
    std::memcpy(&id, opt.tp_id, sizeof(id));
    const ncclResult_t r = nccl().CommInitRank(&comm_, int(tp_), id, int(rank_));
    if (r != ncclSuccess)
      throw WcbError(E_BACKEND, std::string("Backend error: ncclCommInitRank: ") + nccl().GetErrorString(r));
  }
  check(gemv_configure_all(), "configure GEMV kernels");
  check(gemm_tc_configure(), "configure GEMM kernels");
  check(attention_prefill_configure(), "configure prefill attention");
  set_pdl(!(opt.flags & 2));
  try {
    // token embeddings (model.rs:432-446): first name that loads
    bool have_emb = false;
    for (const char* n : {"token_embd.weight", "model.embed_tokens.weight", "embed_tokens.weight"}) {
      const GgufTensor* t = f.find(n);
      if (!t) continue;
      if (t->numel != uint64_t(c.vocab) * c.hidden)
        throw WcbError(E_GENERIC, std::string("tensor ") + n + " has the wrong number of elements");
      std::vector<uint8_t> raw(t->nbytes);
      f.read(*t, raw.data());
      emb_ = static_cast<float*>(dalloc(sizeof(float) * t->numel));
      if (t->dtype == 0) {
        check(cudaMemcpy(emb_, raw.data(), t->nbytes, cudaMemcpyHostToDevice), "upload embeddings");
      } else if (t->dtype == 1) {
        std::vector<float> v(t->numel);
        for (uint64_t i = 0; i < t->numel; ++i) {
          uint16_t hbits;
          std::memcpy(&hbits, &raw[2 * i], 2);
          v[i] = f16_to_f32_host(hbits);
        }
        check(cudaMemcpy(emb_, v.data(), sizeof(float) * v.size(), cudaMemcpyHostToDevice), "upload embeddings");
      } else if (t->dtype == DT_Q4K || t->dtype == DT_Q6K) {
        void* tmp = nullptr;
        check(cudaMalloc(&tmp, t->nbytes), "cudaMalloc");
        check(cudaMemcpy(tmp, raw.data(), t->nbytes, cudaMemcpyHostToDevice), "upload embeddings");
        check(launch_dequant(tmp, int(t->dtype), t->numel / QK_K, emb_, stream_), "dequantise embeddings");
        check(cudaStreamSynchronize(stream_), "dequantise embeddings");
        cudaFree(tmp);
      } else {
        continue;
      }
      have_emb = true;
      break;
    }
    if (!have_emb) throw WcbError(E_PARSE, "Parse error: Missing token embeddings");
    upload_vector(f, "output_norm.weight", c.hidden, 1.0f, out_norm_);

    // LM head (model.rs:482-606)
    bool have_head = false;
    for (const char* n : {"output.weight", "lm_head.weight", "model.lm_head.weight"}) {
      const GgufTensor* t = f.find(n);
      if (!t || (t->dtype != DT_Q4K && t->dtype != DT_Q6K && !dense_dtype(int(t->dtype)))) continue;
      upload_weight(f, n, c.vocab, c.hidden, lm_head_, false, vocab_off_, vocab_l_);
      have_head = true;
      break;
    }
    if (!have_head) {
      // weight tying (model.rs:596-606): the LM head is transpose_matrix(token_embeddings,
      // hidden, vocab), the embedding buffer read as a [hidden][vocab] matrix and
      // transposed to [vocab][hidden] (model.rs:47-55); f32, this rank's vocabulary rows
      const size_t H = c.hidden, V = c.vocab;
      std::vector<float> e(H * V);
      check(cudaMemcpy(e.data(), emb_, sizeof(float) * e.size(), cudaMemcpyDeviceToHost), "read embeddings");
      std::vector<float> head(size_t(vocab_l_) * H);
      for (size_t j = 0; j < vocab_l_; ++j)
        for (size_t i = 0; i < H; ++i) head[j * H + i] = e[i * V + (vocab_off_ + j)];
      lm_head_.dtype = DT_F32;
      lm_head_.rows = vocab_l_;
      lm_head_.cols = uint32_t(H);
      lm_head_.ptr = static_cast<uint8_t*>(dalloc(sizeof(float) * head.size()));
      check(cudaMemcpy(lm_head_.ptr, head.data(), sizeof(float) * head.size(), cudaMemcpyHostToDevice), "LM head");
    }

    const uint32_t kvd = c.kv_heads * hd;
    layers_.resize(c.layers);
    // weight streaming: layer weights to a pinned host copy, streamed through a device ring
    wstream_ = (opt.flags & 16) && tp_ == 1 && c.layers > 0;
    const bool th = wstream_;
    for (uint32_t l = 0; l < c.layers; ++l) {
      DevLayer& L = layers_[l];
      const std::string p = "blk." + std::to_string(l) + ".";
      auto attn = [&](const char* base, uint32_t rows, DevWeight& w, uint32_t row0, uint32_t nrows, uint32_t blk0,
                      uint32_t nblk) {
        std::string n = p + base + ".weight";
        if (!f.find(n)) n = p + base;
        upload_weight(f, n, rows, c.hidden, w, true, row0, nrows, blk0, nblk, th);
      };
      const size_t layer_begin = (wstage_.size() + 255) / 256 * 256;
      // this rank's heads (all of them with one rank)
      attn("attn_q", c.hidden, L.q, rank_ * hq_, hq_, 0, 0);
      attn("attn_k", kvd, L.k, rank_ * kvd_l_, kvd_l_, 0, 0);
      attn("attn_v", kvd, L.v, rank_ * kvd_l_, kvd_l_, 0, 0);
      attn("attn_output", c.hidden, L.o, 0, 0, rank_ * (hq_ / QK_K), hq_ / QK_K);
      upload_weight(f, p + "ffn_gate.weight", c.ffn, c.hidden, L.gate, true, rank_ * ffn_l_, ffn_l_, 0, 0, th);
      upload_weight(f, p + "ffn_up.weight", c.ffn, c.hidden, L.up, true, rank_ * ffn_l_, ffn_l_, 0, 0, th);
      upload_weight(f, p + "ffn_down.weight", c.hidden, c.ffn, L.down, true, 0, 0, rank_ * (ffn_l_ / QK_K),
                    ffn_l_ / QK_K, th);
      if (th) {
        layer_off_.push_back(layer_begin);
        layer_bytes_.push_back(wstage_.size() - layer_begin);
      }
      upload_vector(f, p + "attn_norm.weight", c.hidden, 1.0f, L.attn_norm);
      upload_vector(f, p + "ffn_norm.weight", c.hidden, 1.0f, L.ffn_norm);
      if (L.gate.dtype != L.up.dtype)
        throw WcbError(E_BACKEND, "Backend error: ffn_gate and ffn_up must share a quantisation type");
    }

    if (wstream_) {
      // one pinned host copy of every layer, a ring of wslots_ device slots, and
      // each weight pointed at its place in its layer's slot
      wslots_ = std::min<uint32_t>(2, c.layers);
      for (size_t b : layer_bytes_) wslot_bytes_ = std::max(wslot_bytes_, (b + 255) / 256 * 256);
      check(cudaHostAlloc(reinterpret_cast<void**>(&whost_), std::max<size_t>(wstage_.size(), 16),
                          cudaHostAllocDefault),
            "cudaHostAlloc");
      std::memcpy(whost_, wstage_.data(), wstage_.size());
      std::vector<uint8_t>().swap(wstage_);
      wring_ = static_cast<uint8_t*>(dalloc(wslot_bytes_ * wslots_));
      for (uint32_t l = 0; l < c.layers; ++l) {
        uint8_t* base = wring_ + size_t(l % wslots_) * wslot_bytes_;
        DevLayer& L = layers_[l];
        for (DevWeight* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
          w->ptr = base + (w->host_off - layer_off_[l]);
      }
      check(cudaStreamCreateWithFlags(&cstream_, cudaStreamNonBlocking), "copy stream");
      for (uint32_t i = 0; i < 2; ++i) {
        check(cudaEventCreateWithFlags(&ev_loaded_[i], cudaEventDisableTiming), "event");
        check(cudaEventCreateWithFlags(&ev_free_[i], cudaEventDisableTiming), "event");
      }
    }

    // batched decode slots (generate_batch): each holds its own KV cache, state,
    // sampler history and penalty counts; the tensor-core step needs 128-row
    // tiles that never straddle q / k / v, and 64-row gate / up halves
    // (with tensor parallelism: this rank's q / k / v / gate / up rows)
    bslots_ = !wstream_ ? std::min<uint32_t>(std::max<uint32_t>(opt.max_batch, 1), BATCH_MAX) : 1;
    batch_ok_ = bslots_ > 1 && c.hidden % BATCH_TILE == 0 && hq_ % BATCH_TILE == 0 && kvd_l_ % BATCH_TILE == 0 &&
                ffn_l_ % 64 == 0 && c.heads / c.kv_heads <= 8 && !has_dense_weights();
    (void)kvd;
    if (!batch_ok_) bslots_ = 1;
    // KV cache (kv_cache.rs:6-34), [slot][L][n_kv][max_seq][hd]
    kv_layer_elems_ = size_t(kv_l_) * max_seq_ * hd;
    seq_kv_elems_ = kv_layer_elems_ * c.layers;
    const size_t kv_bytes = seq_kv_elems_ * bslots_ * (opt.kv_half ? 2 : 4);
    kcache_ = dalloc(kv_bytes);
    vcache_ = dalloc(kv_bytes);
    kc_base_ = kcache_;
    vc_base_ = vcache_;
    check(cudaMemset(kcache_, 0, kv_bytes), "clear KV");
    check(cudaMemset(vcache_, 0, kv_bytes), "clear KV");

    build_rope(max_seq_);
    attn_scale_ = 1.0f / std::sqrt(float(hd));  // attention.rs:363

    t_max_ = int(std::min<uint32_t>(T_MAX, std::max<uint32_t>(max_seq_, 1)));
    st_ = static_cast<StepState*>(dalloc(sizeof(StepState) * bslots_));
    check(cudaMemset(st_, 0, sizeof(StepState) * bslots_), "clear state");
    for (uint32_t b = 0; b < bslots_; ++b) {  // bound of the device-side waits (no kernel rewrites it)
      const int wms = int(opt_.wait_ms ? opt_.wait_ms : 2000);
      check(cudaMemcpy(&st_[b].wait_ms, &wms, sizeof(int), cudaMemcpyHostToDevice), "wait bound");
    }
    st_base_ = st_;
    ids_ = static_cast<uint32_t*>(dalloc(sizeof(uint32_t) * std::max<size_t>(max_seq_, 1)));
    hist_cap_ = max_seq_ + 2;
    hist_ = static_cast<uint32_t*>(dalloc(sizeof(uint32_t) * hist_cap_ * bslots_));
    hist_base_ = hist_;
    x_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.hidden));
    h_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.hidden));
    q_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.hidden));
    att_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.hidden));
    act_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.ffn));
    logits_ = static_cast<float*>(dalloc(sizeof(float) * c.vocab));
    if (tp_ > 1) {
      part_y_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_) * c.hidden));
      tpkey_ = static_cast<unsigned long long*>(dalloc(2 * sizeof(unsigned long long)));
      // per-op decode steps: [tp][hidden] partial sums, then [tp][2] LM-head argmax keys;
      // the persistent decode step: [o, down][layer parity][tp][hidden], then [tp][2]
      // (tagged words, written by every rank's peer stores)
      const size_t rn = mk_xofs() + 4 * size_t(tp_) * c.hidden + 2 * size_t(tp_);
      recv_ = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * rn));
      check(cudaMemset(recv_, 0, sizeof(unsigned long long) * rn), "clear receive buffer");
      peers_dev_ = static_cast<unsigned long long**>(dalloc(sizeof(void*) * tp_));
    }
    row_m_ = static_cast<float*>(dalloc(sizeof(float) * size_t(t_max_)));
    xprep_ = static_cast<uint8_t*>(
        dalloc(stage_x_bytes(t_max_, int(std::max({c.hidden, hq_, ffn_l_})))));
    if (tp_ == 1) {  // device sampling: the penalised logits and the random streams
      // per decode slot (the batched step samples every slot at once)
      plog_ = static_cast<float*>(dalloc(sizeof(float) * c.vocab * bslots_));
      rng_ = static_cast<StdRng*>(dalloc(sizeof(StdRng) * bslots_));
      rng_base_ = rng_;
    }
    pen_cnt_ = static_cast<uint32_t*>(dalloc(sizeof(uint32_t) * c.vocab * bslots_));
    check(cudaMemset(pen_cnt_, 0, sizeof(uint32_t) * c.vocab * bslots_), "clear penalty counts");
    pen_base_ = pen_cnt_;
    // attention partials of one decode token split into DECODE_CHUNK-key pieces
    max_splits_ = int((max_seq_ + DECODE_CHUNK - 1) / DECODE_CHUNK);
    part_ = static_cast<float*>(dalloc(sizeof(float) * size_t(c.heads) * max_splits_ * (hd + 2)));
    ticket_ = static_cast<int*>(dalloc(sizeof(int) * size_t(t_max_) * c.kv_heads));
    check(cudaMemset(ticket_, 0, sizeof(int) * size_t(t_max_) * c.kv_heads), "clear tickets");
    check(cudaMallocHost(&host_ids_, sizeof(uint32_t) * std::max<size_t>(max_seq_, 1)), "cudaMallocHost");
    if (batch_ok_) {
      const size_t B = bslots_, H = c.hidden;
      logits_b_ = static_cast<float*>(dalloc(sizeof(float) * B * c.vocab));
      // per-CTA sums of squares of the residual stream: tiles x K slices (<= 8) per sequence
      sqx_ = static_cast<float*>(dalloc(sizeof(float) * B * (H / BATCH_TILE) * 8));
      sqh_ = static_cast<float*>(dalloc(sizeof(float) * B * (H / BATCH_TILE) * 8));
      if (tp_ > 1) tpkeys_b_ = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * 2 * B));
      asplits_ = int((max_seq_ + BATCH_CHUNK - 1) / BATCH_CHUNK);
      apart_ = static_cast<float*>(dalloc(sizeof(float) * B * c.heads * size_t(asplits_) * (hd + 2)));
      aticket_ = static_cast<int*>(dalloc(sizeof(int) * B * c.kv_heads));
      check(cudaMemset(aticket_, 0, sizeof(int) * B * c.kv_heads), "clear tickets");
      check(batch_configure(), "batched decode configure");
    }
    build_decode_step();
    check(cudaDeviceSynchronize(), "load");
  } catch (...) {
    for (void* p : allocs_) cudaFree(p);
    allocs_.clear();
    if (host_ids_) cudaFreeHost(host_ids_);
    host_ids_ = nullptr;
    if (whost_) cudaFreeHost(whost_);
    whost_ = nullptr;
    for (cudaEvent_t& e : ev_loaded_)
      if (e) cudaEventDestroy(e), e = nullptr;
    for (cudaEvent_t& e : ev_free_)
      if (e) cudaEventDestroy(e), e = nullptr;
    if (cstream_) cudaStreamDestroy(cstream_);
    cstream_ = nullptr;
    if (comm_) nccl().CommDestroy(comm_);
    comm_ = nullptr;
    cudaStreamDestroy(stream_);
    stream_ = nullptr;
    throw;
  }
}

Model::~Model() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  if (decode_exec_) cudaGraphExecDestroy(decode_exec_);
  if (decode_graph_) cudaGraphDestroy(decode_graph_);  // graphs holding NCCL calls go before the comm
  if (batch_exec_) cudaGraphExecDestroy(batch_exec_);
  if (batch_graph_) cudaGraphDestroy(batch_graph_);
  // a failed group is aborted, not destroyed: destroying waits for the other ranks
  if (comm_) (tp_failed_ ? nccl().CommAbort : nccl().CommDestroy)(comm_);
  for (void* p : ipc_opened_) cudaIpcCloseMemHandle(p);
  if (cstream_) cudaStreamSynchronize(cstream_);
  for (void* p : allocs_) cudaFree(p);
  if (host_ids_) cudaFreeHost(host_ids_);
  if (whost_) cudaFreeHost(whost_);
  for (cudaEvent_t e : {ev_loaded_[0], ev_loaded_[1], ev_free_[0], ev_free_[1]})
    if (e) cudaEventDestroy(e);
  if (cstream_) cudaStreamDestroy(cstream_);
  if (stream_) cudaStreamDestroy(stream_);
}

// Uploads a 2-D weight [rows][cols] as raw blocks (Q6_K padded to 224 bytes).
// A missing tensor leaves zeros, as the reference's `if let Ok(..)` loads do
// (model.rs:618-760): an all-zero Q4_K block dequantises to 0.
void Model::upload_weight(const GgufFile& f, const std::string& name, uint32_t rows, uint32_t cols, DevWeight& w,
                          bool missing_is_zero, uint32_t row0, uint32_t nrows, uint32_t blk0, uint32_t nblk,
                          bool to_host) {
  // weight streaming: the blocks go to the host copy (256-byte aligned), placed in
  // the device ring once every layer is staged
  auto to_stage = [&](const uint8_t* data, size_t bytes) {
    const size_t off = (wstage_.size() + 255) / 256 * 256;
    wstage_.resize(off + bytes, 0);
    if (data) std::memcpy(wstage_.data() + off, data, bytes);
    w.host_off = off;
    w.ptr = nullptr;
  };
  const size_t nb = size_t(cols) / QK_K;
  if (nrows == 0) nrows = rows - row0;
  if (nblk == 0) nblk = uint32_t(nb) - blk0;
  if (row0 + nrows > rows || blk0 + nblk > nb) throw WcbError(E_GENERIC, "shard outside tensor " + name);
  w.rows = nrows;
  w.cols = nblk * QK_K;
  const GgufTensor* t = f.find(name);
  if (!t) {
    if (!missing_is_zero) throw WcbError(E_GENERIC, "Tensor not found: " + name);
    w.dtype = DT_Q4K;
    const size_t bytes = size_t(nrows) * nblk * Q4K_BYTES;
    if (to_host) {
      to_stage(nullptr, bytes);
      return;
    }
    w.ptr = static_cast<uint8_t*>(dalloc(bytes));
    check(cudaMemset(w.ptr, 0, bytes), "zero weight");
    return;
  }
  if (t->numel != uint64_t(rows) * cols)
    throw WcbError(E_GENERIC, "tensor " + name + " has " + std::to_string(t->numel) + " elements, expected " +
                                  std::to_string(uint64_t(rows) * cols));
  if (t->dtype != DT_Q4K && t->dtype != DT_Q6K && !dense_dtype(int(t->dtype)))
    throw WcbError(E_BACKEND, "Backend error: tensor " + name + " must be F32, F16, Q4_K or Q6_K (GGUF type " +
                                  std::to_string(t->dtype) + ")");
  w.dtype = int(t->dtype);
  // bytes of 256 consecutive values as stored in the file
  const size_t bb = w.dtype == DT_Q4K ? Q4K_BYTES : w.dtype == DT_Q6K ? Q6K_BYTES : dev_block_bytes(w.dtype);
  const size_t row_bytes = nb * bb, take = size_t(nblk) * bb;
  std::vector<uint8_t> raw(size_t(nrows) * take);
  if (take == row_bytes) {
    f.read_range(*t, size_t(row0) * row_bytes, raw.size(), raw.data());  // whole rows: one read
  } else {
    for (uint32_t r = 0; r < nrows; ++r)  // a column slice: part of every row
      f.read_range(*t, size_t(row0 + r) * row_bytes + size_t(blk0) * bb, take, raw.data() + size_t(r) * take);
  }
  if (w.dtype != DT_Q6K) {  // Q4_K, F32, F16: uploaded as read
    if (to_host) {
      to_stage(raw.data(), raw.size());
      return;
    }
    w.ptr = static_cast<uint8_t*>(dalloc(raw.size()));
    check(cudaMemcpy(w.ptr, raw.data(), raw.size(), cudaMemcpyHostToDevice), "upload weight");
  } else {
    const size_t nblock = raw.size() / Q6K_BYTES;
    std::vector<uint8_t> pad(nblock * Q6K_DEV_BYTES, 0);
    for (size_t b = 0; b < nblock; ++b) std::memcpy(&pad[b * Q6K_DEV_BYTES], &raw[b * Q6K_BYTES], Q6K_BYTES);
    if (to_host) {
      to_stage(pad.data(), pad.size());
      return;
    }
    w.ptr = static_cast<uint8_t*>(dalloc(pad.size()));
    check(cudaMemcpy(w.ptr, pad.data(), pad.size(), cudaMemcpyHostToDevice), "upload weight");
  }
}

void Model::issue_layer_copy(uint32_t l) {
  const uint32_t s = l % wslots_;
  check(cudaStreamWaitEvent(cstream_, ev_free_[s], 0), "wait slot");
  check(cudaMemcpyAsync(wring_ + size_t(s) * wslot_bytes_, whost_ + layer_off_[l], layer_bytes_[l],
                        cudaMemcpyHostToDevice, cstream_),
        "stream layer");
  check(cudaEventRecord(ev_loaded_[s], cstream_), "record layer");
}

void Model::all_reduce_sum(float* buf, size_t n) {
  const ncclResult_t r = nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, comm_, stream_);
  if (r != ncclSuccess) throw WcbError(E_BACKEND, std::string("Backend error: ncclAllReduce: ") + nccl().GetErrorString(r));
}

void Model::upload_vector(const GgufFile& f, const std::string& name, uint32_t n, float fill, float*& dst) {
  std::vector<float> v(n, fill);
  const GgufTensor* t = f.find(name);
  if (t && (t->dtype == 0 || t->dtype == 1)) {
    if (t->numel != n)
      throw WcbError(E_GENERIC, "tensor " + name + " has " + std::to_string(t->numel) + " elements, expected " +
                                    std::to_string(n));
    std::vector<uint8_t> raw(t->nbytes);
    f.read(*t, raw.data());
    for (uint32_t i = 0; i < n; ++i) {
      if (t->dtype == 0) {
        std::memcpy(&v[i], &raw[4 * size_t(i)], 4);
      } else {
        uint16_t hb;
        std::memcpy(&hb, &raw[2 * size_t(i)], 2);
        v[i] = f16_to_f32_host(hb);
      }
    }
  }
  dst = static_cast<float*>(dalloc(sizeof(float) * n));
  check(cudaMemcpy(dst, v.data(), sizeof(float) * n, cudaMemcpyHostToDevice), "upload vector");
}

// cos / sin of the RoPE angles exactly as apply_rope computes them
// (attention.rs:230-248): freq = 1 / theta^(i/hd) and angle = pos * freq in f32.
void Model::build_rope(uint32_t len) {
  const uint32_t hd = cfg_.head_dim(), half = hd / 2;
  std::vector<float> cs(size_t(len) * half), sn(size_t(len) * half);
  for (uint32_t i = 0; i < hd; i += 2) {
    const float freq = 1.0f / std::pow(cfg_.theta, float(i) / float(hd));
    for (uint32_t p = 0; p < len; ++p) {
      const float angle = float(p) * freq;
      cs[size_t(p) * half + i / 2] = std::cos(angle);
      sn[size_t(p) * half + i / 2] = std::sin(angle);
    }
  }
  float* c = static_cast<float*>(dalloc(sizeof(float) * cs.size()));
  float* s = static_cast<float*>(dalloc(sizeof(float) * sn.size()));
  check(cudaMemcpy(c, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice), "upload rope");
  check(cudaMemcpy(s, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice), "upload rope");
  rope_cos_ = c;
  rope_sin_ = s;
  rope_len_ = len;
  if (decode_exec_) {  // captured graphs hold the old table pointers
    cudaGraphExecDestroy(decode_exec_);
    cudaGraphDestroy(decode_graph_);
    decode_exec_ = nullptr;
    decode_graph_ = nullptr;
  }
}

void Model::set_state(int position, int kv_len, int n_tokens) {
  ++mk_launches_;  // the state kernel advances the epoch too
  check(launch_set_state(st_, position, kv_len, n_tokens, stream_), "set state");
}

void Model::gemv(const DevWeight* segs, int nseg, int K, int M, const float* x, int ldx, const float* norm_w,
                 float eps, int pro, int epi, float* y, int ldy, const float* resid, int ldr, float* q, int ldq,
                 int layer, int token_offset) {
  // one launch per run of segments sharing a quantisation type (a Q4_K_M layer
  // can mix Q4_K q/k with a Q6_K v)
  int row_offset = 0;
  for (int s0 = 0; s0 < nseg;) {
    int s1 = s0 + 1;
    if (epi == EPI_SWIGLU) s1 = nseg;
    else
      while (s1 < nseg && segs[s1].dtype == segs[s0].dtype) ++s1;
    GemvArgs a{};
    int rows = 0;
    for (int i = s0; i < s1; ++i) {
      a.seg[i - s0].w = segs[i].ptr;
      a.seg[i - s0].dtype = segs[i].dtype;
      a.seg[i - s0].rows = int(segs[i].rows);
      rows += int(segs[i].rows);
    }
    a.nseg = s1 - s0;
    a.K = K;
    a.ngroups = epi == EPI_SWIGLU ? int(segs[0].rows) / 2 : rows / 4;
    a.norm_w = norm_w;
    a.eps = eps;
    a.ldx = ldx;
    a.ldy = ldy;
    a.ldr = ldr;
    a.ldq = ldq;
    a.hidden = int(hq_);     // query rows of the [q; k; v] segments held here
    a.kv_dim = int(kvd_l_);
    a.head_dim = int(cfg_.head_dim());
    a.max_seq = int(max_seq_);
    a.kv_half = int(opt_.kv_half);
    a.row_offset = row_offset;
    if (layer >= 0) {
      const size_t esz = opt_.kv_half ? 2 : 4;
      a.kc = static_cast<uint8_t*>(kcache_) + size_t(layer) * kv_layer_elems_ * esz;
      a.vc = static_cast<uint8_t*>(vcache_) + size_t(layer) * kv_layer_elems_ * esz;
    }
    a.rope_cos = rope_cos_;
    a.rope_sin = rope_sin_;
    a.st = st_;
    a.gen_mode = gen_mode_;
    a.vocab_off = int(vocab_off_);
    a.peers = peers_dev_;
    a.tp_rank = int(rank_);
    a.tp_size = int(tp_);
    a.peer_phase = peer_phase_;
    a.pen_cnt = pen_cnt_;
    a.pen_cnt_w = pen_cnt_;
    a.rep = rep_;
    a.hist = hist_;
    a.pdl = 1;
    if (M >= TC_MIN_TOKENS && epi != EPI_LMHEAD && !(opt_.flags & 4) && !dense_dtype(segs[s0].dtype)) {
      // prefill: one tensor-core GEMM over all M tokens
      GemvArgs b = a;
      b.M = M;
      b.x = x;
      b.y = y;
      b.resid = resid;
      b.q = q;
      b.token_offset = token_offset;
      if (pro == PRO_RMSNORM) {
        check(launch_row_rms(x, ldx, M, K, eps, row_m_, true, stream_), "row rms");
        ++launches_;
      }
      // the activations once as the GEMM's fp16 hi / lo A tiles, shared by all row tiles
      check(launch_stage_x(x, ldx, M, K, pro == PRO_RMSNORM ? norm_w : nullptr, xprep_, stream_), "stage x");
      ++launches_;
      b.xprep = xprep_;
      check(launch_gemm_tc(b, pro, epi, row_m_, stream_), "gemm");
      ++launches_;
      row_offset += rows;
      s0 = s1;
      continue;
    }
    const int mmax = epi == EPI_LMHEAD ? 1 : dense_dtype(segs[s0].dtype) ? 4 : gemv_max_cols(K);
    for (int c0 = 0; c0 < M; c0 += mmax) {
      GemvArgs b = a;
      b.M = std::min(mmax, M - c0);
      b.x = x + size_t(c0) * ldx;
      b.y = y ? y + size_t(c0) * ldy : nullptr;
      b.resid = resid ? resid + size_t(c0) * ldr : nullptr;
      b.q = q ? q + size_t(c0) * ldq : nullptr;
      b.token_offset = token_offset + c0;
      check(launch_gemv(b, pro, epi, stream_), "gemv");
      ++launches_;
    }
    row_offset += rows;
    s0 = s1;
  }
}

void Model::enqueue_layers(int T, bool decode) {
  // decode steps of a connected tensor-parallel group exchange partial sums by
  // peer stores; prefill chunks and forward() use NCCL (whose collectives also
  // order the ranks before the first peer store of a session)
  const bool peer = tp_ > 1 && p2p_ && decode && T == 1;
  const ModelConfig& c = cfg_;
  const int H = int(c.hidden), hd = int(c.head_dim());
  const int HQ = int(hq_), FL = int(ffn_l_);
  if (wstream_ && !wprimed_) {
    for (uint32_t l = 0; l < wslots_; ++l) issue_layer_copy(l);
    wprimed_ = true;
  }
  for (uint32_t l = 0; l < c.layers; ++l) {
    const DevLayer& L = layers_[l];
    if (wstream_) check(cudaStreamWaitEvent(stream_, ev_loaded_[l % wslots_], 0), "wait layer");
    // RMSNorm(eps 1e-6, layer.rs:51-57) -> Q/K/V projections (attention.rs:80-129)
    // -> RoPE (:140-143) -> KV append (:162); this rank's heads only
    const DevWeight qkv[3] = {L.q, L.k, L.v};
    gemv(qkv, 3, H, T, x_, H, L.attn_norm, 1e-6f, PRO_RMSNORM, EPI_QKV, nullptr, 0, nullptr, 0, q_, HQ, int(l), 0);
    // attention over the cache (attention.rs:173, :332-435)
    AttnArgs a{};
    a.q = q_;
    const size_t esz = opt_.kv_half ? 2 : 4;
    a.kc = static_cast<uint8_t*>(kcache_) + size_t(l) * kv_layer_elems_ * esz;
    a.vc = static_cast<uint8_t*>(vcache_) + size_t(l) * kv_layer_elems_ * esz;
    a.kv_half = int(opt_.kv_half);
    a.out = att_;
    a.part = part_;
    a.ticket = ticket_;
    a.n_heads = int(heads_l_);
    a.n_kv = int(kv_l_);
    a.head_dim = hd;
    a.max_seq = int(max_seq_);
    a.T = T;
    if (T == 1) {  // decode: split the keys for parallelism, merged by the last CTA
      a.chunk = DECODE_CHUNK;
      a.max_splits = max_splits_;
    } else {  // prefill: the query tokens give the parallelism, one split per token
      a.chunk = int(max_seq_);
      a.max_splits = 1;
    }
    a.scale = attn_scale_;
    a.st = st_;
    if (T >= TC_MIN_TOKENS && !(opt_.flags & 4) && attention_prefill_supported(a.n_heads, a.n_kv, hd))
      check(launch_attention_prefill(a, stream_), "attention");  // prefill chunk: tensor cores
    else
      check(launch_attention(a, stream_), "attention");
    ++launches_;
    // output projection + residual (attention.rs:182-191, layer.rs:68); with several
    // ranks each holds the columns of its heads: partial sums, all-reduced
    const DevWeight o[1] = {L.o};
    if (tp_ == 1) {
      gemv(o, 1, HQ, T, att_, HQ, nullptr, 0.0f, PRO_NONE, EPI_RESID, h_, H, x_, H, nullptr, 0, -1, 0);
    } else if (peer) {
      peer_phase_ = int(2 * l);
      gemv(o, 1, HQ, T, att_, HQ, nullptr, 0.0f, PRO_NONE, EPI_PEER, nullptr, H, nullptr, 0, nullptr, 0, -1, 0);
      check(launch_tp_reduce_add(h_, x_, recv_, int(tp_), size_t(H), int(2 * l), st_, stream_), "peer reduce");
      launches_ += 1;
    } else {
      gemv(o, 1, HQ, T, att_, HQ, nullptr, 0.0f, PRO_NONE, EPI_STORE, part_y_, H, nullptr, 0, nullptr, 0, -1, 0);
      all_reduce_sum(part_y_, size_t(T) * H);
      check(launch_add(h_, x_, part_y_, size_t(T) * H, st_, stream_), "residual");
      launches_ += 1;
    }
    // RMSNorm(eps 1e-6, layer.rs:71-77) -> gate/up -> SwiGLU (ffn.rs:60-94)
    const DevWeight gu[2] = {L.gate, L.up};
    gemv(gu, 2, H, T, h_, H, L.ffn_norm, 1e-6f, PRO_RMSNORM, EPI_SWIGLU, act_, FL, nullptr, 0, nullptr, 0, -1, 0);
    // down projection + residual (ffn.rs:97-106, layer.rs:86)
    const DevWeight dn[1] = {L.down};
    if (tp_ == 1) {
      gemv(dn, 1, FL, T, act_, FL, nullptr, 0.0f, PRO_NONE, EPI_RESID, x_, H, h_, H, nullptr, 0, -1, 0);
    } else if (peer) {
      peer_phase_ = int(2 * l + 1);
      gemv(dn, 1, FL, T, act_, FL, nullptr, 0.0f, PRO_NONE, EPI_PEER, nullptr, H, nullptr, 0, nullptr, 0, -1, 0);
      check(launch_tp_reduce_add(x_, h_, recv_, int(tp_), size_t(H), int(2 * l + 1), st_, stream_), "peer reduce");
      launches_ += 1;
    } else {
      gemv(dn, 1, FL, T, act_, FL, nullptr, 0.0f, PRO_NONE, EPI_STORE, part_y_, H, nullptr, 0, nullptr, 0, -1, 0);
      all_reduce_sum(part_y_, size_t(T) * H);
      check(launch_add(x_, h_, part_y_, size_t(T) * H, st_, stream_), "residual");
      launches_ += 1;
    }
    if (wstream_) {  // the slot is free once this layer's kernels ran; refill it ahead
      check(cudaEventRecord(ev_free_[l % wslots_], stream_), "free slot");
      if (l + wslots_ < c.layers) issue_layer_copy(l + wslots_);
    }
  }
  if (wstream_)  // the next forward's first layers, behind this one's last users of their slots
    for (uint32_t l = 0; l < wslots_; ++l) issue_layer_copy(l);
}

// final RMSNorm with the config eps (model.rs:937-943) + LM head on the last
// token (model.rs:975-1037); in generate mode the same launch applies the
// repetition penalty, takes the argmax and does generate()'s bookkeeping
void Model::enqueue_lm_head(int T, bool gen) {
  const int H = int(cfg_.hidden);
  const DevWeight head[1] = {lm_head_};
  // with several ranks each scores its vocabulary rows; the argmax key (order-
  // preserving logit bits | token id) and the NaN flag are max-reduced over the
  // ranks, then every rank runs the same sampler bookkeeping
  const bool dev_sample = gen && sample_mode_ != 0;
  gen_mode_ = (gen && !dev_sample) ? (tp_ > 1 ? 2 : 1) : 0;
  gemv(head, 1, H, 1, x_ + size_t(T - 1) * H, H, out_norm_, cfg_.eps, PRO_RMSNORM, EPI_LMHEAD, logits_,
       int(cfg_.vocab), nullptr, 0, nullptr, 0, -1, 0);
  gen_mode_ = 0;
  if (dev_sample) enqueue_sampler();
  if (gen && tp_ > 1 && p2p_) {
    // the argmax keys exchanged by peer stores too: a decode step then makes no NCCL
    // call, so every wait on another rank in it is bounded
    check(launch_tp_key_exchange(st_, peers_dev_, recv_, int(rank_), int(tp_), size_t(tp_) * cfg_.hidden, hist_,
                                 pen_cnt_, stream_),
          "argmax key exchange");
    ++launches_;
  } else if (gen && tp_ > 1) {
    check(launch_tp_pack_key(st_, tpkey_, stream_), "argmax key");
    const ncclResult_t r = nccl().AllReduce(tpkey_, tpkey_, 2, ncclUint64, ncclMax, comm_, stream_);
    if (r != ncclSuccess) throw WcbError(E_BACKEND, std::string("Backend error: ncclAllReduce: ") + nccl().GetErrorString(r));
    check(launch_tp_finish(st_, tpkey_, hist_, pen_cnt_, stream_), "sampler bookkeeping");
    launches_ += 2;
  }
}

// penalty, top-k / top-p draw and generate()'s bookkeeping on the device
void Model::enqueue_sampler() {
  if (sample_mode_ == 1)  // 1 <= top_k <= 1024
    check(launch_sample(logits_, plog_, int(cfg_.vocab), st_, hist_, pen_cnt_, rep_, samp_t_, samp_k_, samp_tp_, rng_,
                        stream_),
          "sampler");
  else  // every other sampled configuration
    check(launch_sample_full(logits_, plog_, int(cfg_.vocab), st_, hist_, pen_cnt_, rep_, samp_t_, samp_k_, samp_tp_,
                             rng_, nullptr, stream_),
          "sampler");
  ++launches_;
}

void Model::enqueue_forward(const uint32_t* dev_ids, int T, bool from_hist) {
  if (from_hist) check(launch_embed_last(emb_, int(cfg_.vocab), int(cfg_.hidden), hist_, x_, st_, stream_), "embed");
  else check(launch_embed(emb_, int(cfg_.vocab), int(cfg_.hidden), dev_ids, T, x_, st_, stream_), "embed");
  ++launches_;
  enqueue_layers(T, from_hist);
}

void Model::tp_ipc_handle(void* out) const {
  if (tp_ < 2) throw WcbError(E_INVALID, "Invalid argument: the model is not tensor-parallel");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, recv_);
  if (e != cudaSuccess) throw WcbError(E_BACKEND, std::string("Backend error: cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(out, &h, sizeof(h));
}

void Model::tp_connect(const uint8_t* handles, uint32_t n) {
  if (tp_ < 2 || n != tp_) throw WcbError(E_INVALID, "Invalid argument: one IPC handle per tensor-parallel rank");
  check(cudaSetDevice(device_), "cudaSetDevice");
  std::vector<unsigned long long*> ptrs(tp_);
  for (uint32_t r = 0; r < tp_; ++r) {
    if (r == rank_) {
      ptrs[r] = recv_;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + 64 * size_t(r), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      throw WcbError(E_BACKEND, std::string("Backend error: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    ipc_opened_.push_back(p);
    ptrs[r] = static_cast<unsigned long long*>(p);
  }
  check(cudaMemcpy(peers_dev_, ptrs.data(), sizeof(void*) * tp_, cudaMemcpyHostToDevice), "peer table");
  p2p_ = true;
  if (decode_exec_) {  // re-capture the decode step with the peer exchange
    cudaGraphExecDestroy(decode_exec_);
    cudaGraphDestroy(decode_graph_);
    decode_exec_ = nullptr;
    decode_graph_ = nullptr;
  }
}

void Model::tp_abort() {
  tp_failed_ = true;
  if (comm_) {
    nccl().CommAbort(comm_);
    comm_ = nullptr;
  }
}

void Model::check_group() const {
  if (tp_failed_)
    throw WcbError(E_BACKEND, "Backend error: the tensor-parallel group has failed (a rank stopped or the group "
                              "was aborted); free this model and load the group again");
}

void Model::forward(const uint32_t* ids, size_t n, size_t position, float* logits_out) {
  check_group();
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (n == 0) throw WcbError(E_INVALID, "Invalid tensor shape: empty token sequence");
  if (kv_len_ + n > max_seq_)
    throw WcbError(E_PARSE, "Parse error: KV cache overflow: " + std::to_string(kv_len_) + " + " + std::to_string(n) +
                                " > " + std::to_string(max_seq_));
  if (position + n > rope_len_) build_rope(uint32_t(std::max<size_t>(position + n, size_t(rope_len_) * 2)));
  std::memcpy(host_ids_, ids, n * sizeof(uint32_t));
  check(cudaMemcpyAsync(ids_, host_ids_, n * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_), "upload ids");
  if (n == 1 && use_mk()) {  // one token: the persistent decode step
    set_state(int(position), int(kv_len_), 1);
    launch_decode_step_kernel(0);
  } else {
    for (size_t c0 = 0; c0 < n; c0 += size_t(t_max_)) {
      const int T = int(std::min(n - c0, size_t(t_max_)));
      set_state(int(position + c0), int(kv_len_ + c0), T);
      enqueue_forward(ids_ + c0, T, false);
    }
    const int last_T = int(n - ((n - 1) / size_t(t_max_)) * size_t(t_max_));
    enqueue_lm_head(last_T, false);
  }
  if (logits_out)  // with several ranks: this rank's vocabulary slice only
    check(cudaMemcpyAsync(logits_out + vocab_off_, logits_, sizeof(float) * vocab_l_, cudaMemcpyDeviceToHost,
                          stream_),
          "download logits");
  check(cudaStreamSynchronize(stream_), "forward");
  {
    // bounded device waits that expired: 4 / 8 in the persistent decode step, 16 in
    // the tensor-parallel exchange (a rank stopped sending its partial sums)
    int err = 0;
    check(cudaMemcpy(&err, &st_->err, sizeof(int), cudaMemcpyDeviceToHost), "read state");
    if (err & 16) tp_failed_ = true;  // the ranks' exchange epochs no longer agree
    if (err & 28)
      throw WcbError(E_BACKEND, std::string("Backend error: ") +
                                    (err & 16 ? "tensor-parallel exchange" : "decode step kernel") +
                                    ": a bounded wait expired (device error word " + std::to_string(err) + ")");
  }
  kv_len_ += n;
}

// Phase list of the persistent decode step: per layer [q;k;v] (one part per
// run of equal quantisation types), attention, o, gate/up, down; then the LM
// head. Each phase waits on the counter of the phase whose output it reads.
void Model::build_decode_step() {
  mk_ok_ = false;
  // weight streaming and dense (F32 / F16) weights run the per-op kernels
  if ((opt_.flags & 8) || wstream_ || has_dense_weights()) return;
  if (decode_step_configure() != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  const ModelConfig& c = cfg_;
  // this rank's shard: all hidden rows of o / down, its query / KV heads and FFN rows
  const int H = int(c.hidden), F = int(ffn_l_), HQ = int(hq_);
  std::vector<MkPart> parts;
  int phase = 0, prev_d = -1;
  bool too_many = false;  // 4-row groups of a part are counted in 16 bits
  auto groups = [&](size_t n) {
    too_many |= n > 65535 || n == 0;
    return uint16_t(n);
  };
  for (uint32_t l = 0; l < c.layers; ++l) {
    const DevLayer& L = layers_[l];
    const int p_qkv = phase++;
    const DevWeight* segs[3] = {&L.q, &L.k, &L.v};
    const size_t first = parts.size();
    int row_off = 0;
    for (int s0 = 0; s0 < 3;) {
      int s1 = s0 + 1;
      while (s1 < 3 && segs[s1]->dtype == segs[s0]->dtype) ++s1;
      MkPart P{};
      P.kind = MK_QKV;
      P.dtype = uint8_t(segs[s0]->dtype);
      P.K = H;
      int rows = 0;
      for (int i = s0; i < s1; ++i) {
        P.w[i - s0] = segs[i]->ptr;
        if (i - s0 == 0) P.rows0 = int(segs[i]->rows);
        if (i - s0 == 1) P.rows1 = int(segs[i]->rows);
        rows += int(segs[i]->rows);
      }
      P.nseg = uint8_t(s1 - s0);
      P.ngroups = groups(size_t(rows) / 4);
      P.row_offset = row_off;
      row_off += rows;
      P.phase = int16_t(p_qkv);
      P.dep = int16_t(prev_d);
      P.norm = L.attn_norm;
      P.eps = 1e-6f;
      parts.push_back(P);
      s0 = s1;
    }
    parts[first].first = 1;
    const int p_att = phase++;
    {
      MkPart P{};
      P.kind = MK_ATT;
      P.phase = int16_t(p_att);
      P.dep = int16_t(p_qkv);
      P.first = 1;
      parts.push_back(P);
    }
    const int p_o = phase++;
    {
      MkPart P{};
      P.kind = MK_O;
      P.dtype = uint8_t(L.o.dtype);
      P.K = HQ;
      P.w[0] = L.o.ptr;
      P.rows0 = int(L.o.rows);
      P.nseg = 1;
      P.ngroups = groups(L.o.rows / 4);
      P.phase = int16_t(p_o);
      P.dep = int16_t(p_att);
      P.first = 1;
      parts.push_back(P);
    }
    if (L.gate.dtype != L.up.dtype) return;  // gate/up rows are paired inside one tile
    const int p_gu = phase++;
    {
      MkPart P{};
      P.kind = MK_GU;
      P.dtype = uint8_t(L.gate.dtype);
      P.K = H;
      P.w[0] = L.gate.ptr;
      P.w[1] = L.up.ptr;
      P.rows0 = int(L.gate.rows);
      P.rows1 = int(L.up.rows);
      P.nseg = 2;
      P.ngroups = groups(L.gate.rows / 2);
      P.phase = int16_t(p_gu);
      P.dep = int16_t(p_o);
      P.norm = L.ffn_norm;
      P.eps = 1e-6f;
      P.first = 1;
      parts.push_back(P);
    }
    const int p_d = phase++;
    {
      // an input longer than the step's limb planes (the 70B width's FFN, 28672) is cut
      // into a K chain of parts over 8-block chunks; their partial sums meet per group
      const int nb = F / QK_K, np = (F + MK_MAX_INPUT - 1) / MK_MAX_INPUT;
      const int per = ((nb + np - 1) / np + 7) / 8 * 8;  // blocks of a part, whole 8-block chunks
      const size_t bb = dev_block_bytes(L.down.dtype);
      for (int b0 = 0; b0 < nb; b0 += per) {
        const int b1 = std::min(nb, b0 + per);
        MkPart P{};
        P.kind = MK_D;
        P.dtype = uint8_t(L.down.dtype);
        P.K = (b1 - b0) * QK_K;
        P.w[0] = L.down.ptr + size_t(b0) * bb;
        P.rows0 = int(L.down.rows);
        P.nseg = 1;
        P.ngroups = groups(L.down.rows / 4);
        P.phase = int16_t(p_d);
        P.dep = int16_t(p_gu);
        P.first = 1;
        if (np > 1) {
          P.kofs = b0 * QK_K;
          P.row_stride = int(size_t(nb) * bb);
          P.kch0 = int16_t(b0 / 8);
          P.kchs = int16_t((nb + 7) / 8);
          P.kchain = uint8_t(b1 < nb ? 1 : 2);
        }
        parts.push_back(P);
      }
    }
    prev_d = p_d;
  }
  {
    MkPart P{};
    P.kind = MK_LM;
    P.dtype = uint8_t(lm_head_.dtype);
    P.K = H;
    P.w[0] = lm_head_.ptr;
    P.rows0 = int(lm_head_.rows);
    P.nseg = 1;
    P.ngroups = groups(lm_head_.rows / 4);
    P.phase = int16_t(phase++);
    P.dep = int16_t(prev_d);
    P.norm = out_norm_;
    P.eps = c.eps;
    P.first = 1;
    parts.push_back(P);
  }
  if (phase > 1023) return;  // tags hold the phase in 10 bits
  MkArgs a{};
  a.n_kv = int(kv_l_);
  a.n_heads = int(heads_l_);
  a.head_dim = int(c.head_dim());
  a.kv_half = int(opt_.kv_half);  // selects the kernel instantiation the plan checks
  a.hidden = H;
  a.qdim = HQ;
  a.tp_size = int(tp_);
  a.tp_rank = int(rank_);
  if (too_many) return;
  if (!decode_step_plan(parts.data(), int(parts.size()), a, int(c.heads / c.kv_heads), &mk_smem_)) return;
  auto upload = [&](const void* src, size_t bytes) {
    void* d = dalloc(bytes);
    check(cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice), "upload step plan");
    return d;
  };
  a.parts = static_cast<const MkPart*>(upload(parts.data(), sizeof(MkPart) * parts.size()));
  a.st = st_;
  a.emb = emb_;
  a.vocab = int(c.vocab);
  a.ffn = F;
  a.max_seq = int(max_seq_);
  a.kcache = kcache_;
  a.vcache = vcache_;
  a.kv_layer_elems = kv_layer_elems_;
  a.kv_half = int(opt_.kv_half);
  a.attn_scale = attn_scale_;
  const size_t kvd = kvd_l_;
  // xa, xb, q, att (one row per key split), the splits' (max, sum), act, knew, vnew
  const size_t smax = size_t(a.att_smax);
  const size_t tagged = (3 + smax) * size_t(H) + smax * heads_l_ * 2 + size_t(F) + 2 * kvd;
  unsigned long long* t = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * tagged));
  check(cudaMemset(t, 0, sizeof(unsigned long long) * tagged), "clear activations");
  mk_tagged_ = t;
  mk_tagged_n_ = tagged;
  a.xa = t;
  a.xb = a.xa + H;
  a.q = a.xb + H;
  a.att = a.q + H;
  a.attml = a.att + smax * H;
  a.act = a.attml + smax * heads_l_ * 2;
  a.knew = a.act + F;
  a.vnew = a.knew + kvd;
  a.logits = logits_;
  float* zero = static_cast<float*>(dalloc(sizeof(float) * H));
  check(cudaMemset(zero, 0, sizeof(float) * H), "clear zero row");
  a.zero = zero;
  a.ids = ids_;
  a.hist = hist_;
  a.pen_cnt = pen_cnt_;
  a.vocab_off = int(vocab_off_);
  a.peers = peers_dev_;  // filled by tp_connect
  a.xofs = mk_xofs();
  mk_ = a;
  mk_ok_ = true;
}

void Model::launch_decode_step_kernel(int gen_mode) {
  if (++mk_launches_ >= (1u << 21)) {
    // tags are epoch * 1024 + phase + 1 in 32 bits: restart the epochs well
    // before they wrap (no launch is in flight after these stream-ordered clears)
    check(cudaMemsetAsync(mk_tagged_, 0, sizeof(unsigned long long) * mk_tagged_n_, stream_), "clear activations");
    check(cudaMemsetAsync(&st_->epoch, 0, sizeof(int), stream_), "clear epoch");
    mk_launches_ = 0;
  }
  MkArgs a = mk_;
  a.rope_cos = rope_cos_;
  a.rope_sin = rope_sin_;
  a.gen_mode = gen_mode;
  a.rep = rep_;
  // test hook for the bounded waits (unset in normal use): withhold one phase's outputs
  const char* drop = std::getenv("WCB_TEST_DROP_PHASE");
  a.drop_phase = drop && *drop ? std::atoi(drop) : -1;
  check(launch_decode_step(a, mk_smem_, stream_), "decode step");
}

void Model::decode_steps(int steps) {
  for (int i = 0; i < steps; ++i) {
    if (use_mk()) {  // the single-launch step (+ the device sampler of a sampled config)
      launch_decode_step_kernel(sample_mode_ == 0 ? 1 : 2);
      if (sample_mode_ != 0) enqueue_sampler();
    } else if (decode_exec_) {
      check(cudaGraphLaunch(decode_exec_, stream_), "graph launch");
    } else {
      enqueue_forward(nullptr, 1, true);
      enqueue_lm_head(1, true);
    }
  }
}

void Model::capture_decode_graph() {
  cudaGraph_t g = nullptr;
  launches_ = 0;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    enqueue_forward(nullptr, 1, true);
    enqueue_lm_head(1, true);
  } catch (...) {
    cudaStreamEndCapture(stream_, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  check(cudaStreamEndCapture(stream_, &g), "end capture");
  cudaGraphExec_t e = nullptr;
  const cudaError_t r = cudaGraphInstantiate(&e, g, 0);
  if (r != cudaSuccess) {
    cudaGraphDestroy(g);
    check(r, "graph instantiate");
  }
  decode_graph_ = g;
  decode_exec_ = e;
  launches_per_step_ = launches_;
}

void Model::start(const uint32_t* prompt, size_t n, const GenParams& g) {
  check_group();
  check(cudaSetDevice(device_), "cudaSetDevice");
  ++session_;
  sess_active_ = false;
  clear_kv();  // model.rs:1344
  if (n == 0) throw WcbError(E_PARSE, "Parse error: Empty token sequence");
  sess_params_ = g;
  sess_sampler_ = std::make_unique<Sampler>(g.seed, g.temperature, g.top_p, g.top_k, g.repetition_penalty);
  sess_greedy_ = sess_sampler_->greedy();
  if (!sess_greedy_ && tp_ > 1)  // the host sampler would need every rank's logits
    throw WcbError(E_BACKEND, "Backend error: sampled decoding (temperature > 0) with tensor parallelism");
  sess_delivered_ = 0;
  sess_tokens_.clear();
  sess_done_ = false;
  sess_steps_left_ = g.max_tokens > 1 ? size_t(g.max_tokens) - 1 : 0;
  // sampled decoding runs on the device (sample_dev.cu; the host sampler's order of
  // operations, so a seed draws the same tokens): the same device-driven loop as
  // greedy decoding. Mode 1: 1 <= top_k <= 1024; mode 2: every other configuration.
  // Load flag bit 5 keeps the host sampler (each step's logits copied back).
  const bool dev_sample = !sess_greedy_ && plog_ && !(opt_.flags & 32);
  sess_host_ = !sess_greedy_ && !dev_sample;
  sample_mode_ = dev_sample ? (sess_sampler_->fixed_path(cfg_.vocab) ? 1 : 2) : 0;
  if (dev_sample) {
    samp_t_ = sess_sampler_->temperature();
    samp_k_ = int(sess_sampler_->top_k());
    samp_tp_ = sess_sampler_->top_p();
    const StdRng seed = sess_sampler_->seed_state();
    check(cudaMemcpyAsync(rng_, &seed, sizeof(seed), cudaMemcpyHostToDevice, stream_), "seed");
    check(cudaStreamSynchronize(stream_), "seed");
  }
  if (sess_host_) {
    // host-sampled path: Model::generate's loop with the LogitsProcessor on the host
    std::vector<float> logits(cfg_.vocab);
    for (size_t cs = 0; cs < n; cs += size_t(t_max_)) {
      const size_t ce = std::min(cs + size_t(t_max_), n);
      forward(prompt + cs, ce - cs, cs, ce == n ? logits.data() : nullptr);
    }
    sess_last_ = sess_sampler_->sample(logits.data(), logits.size());  // no EOS check (model.rs:1380)
    sess_tokens_.push_back(sess_last_);
    sess_done_ = sess_steps_left_ == 0;
    sess_active_ = true;
    return;
  }
  // greedy: the decode loop runs on the device (argmax + repetition penalty +
  // EOS / max_tokens bookkeeping in the sampler kernel), no host round trip per token
  prefill_greedy(prompt, n, g);
  const float rep = g.repetition_penalty;
  const bool same_graph = graph_rep_ == rep && graph_mode_ == sample_mode_ &&
                          (sample_mode_ == 0 || (graph_t_ == samp_t_ && graph_k_ == samp_k_ && graph_tp_ == samp_tp_));
  if (use_mk()) {
    launches_per_step_ = sample_mode_ == 0 ? 1 : 2;
  } else if (!(opt_.flags & 1) && !wstream_ && (!decode_exec_ || !same_graph)) {
    if (decode_exec_) {
      cudaGraphExecDestroy(decode_exec_);
      cudaGraphDestroy(decode_graph_);
      decode_exec_ = nullptr;
      decode_graph_ = nullptr;
    }
    graph_rep_ = rep;
    capture_decode_graph();
  }
  graph_rep_ = rep;
  graph_mode_ = sample_mode_;
  graph_t_ = samp_t_;
  graph_k_ = samp_k_;
  graph_tp_ = samp_tp_;
  sync_session_state();
  sess_active_ = true;
}

void Model::sync_session_state() {
  check(cudaMemcpyAsync(&sess_state_, st_, sizeof(StepState), cudaMemcpyDeviceToHost, stream_), "read state");
  check(cudaStreamSynchronize(stream_), "generate");
  kv_len_ = size_t(sess_state_.kv_len);
  if (sess_state_.err & 28) {
    sess_done_ = true;
    if (sess_state_.err & 16) tp_failed_ = true;
    throw WcbError(E_BACKEND, std::string("Backend error: ") +
                                  (sess_state_.err & 16 ? "tensor-parallel exchange" : "decode step kernel") +
                                  ": a bounded wait expired (device error word " + std::to_string(sess_state_.err) +
                                  ")");
  }
  if (sess_state_.err & 1) {
    sess_done_ = true;
    throw WcbError(E_GENERIC, "Runtime error: NaN logit");
  }
  if (sess_state_.done) sess_done_ = true;
}

std::vector<uint32_t> Model::next(size_t max_tokens, bool* finished) {
  if (!sess_active_) throw WcbError(E_INVALID, "Invalid argument: no active generation on this model");
  check_group();
  check(cudaSetDevice(device_), "cudaSetDevice");
  std::vector<uint32_t> out;
  if (sess_host_) {
    std::vector<float> logits(cfg_.vocab);
    while (sess_tokens_.size() - sess_delivered_ < max_tokens && !sess_done_) {
      if (sess_steps_left_ == 0) { sess_done_ = true; break; }
      forward(&sess_last_, 1, kv_len_, logits.data());
      const uint32_t nx = sess_sampler_->sample(logits.data(), logits.size());
      --sess_steps_left_;
      if (nx == sess_params_.eos) { sess_done_ = true; break; }
      sess_tokens_.push_back(nx);
      sess_last_ = nx;
      if (sess_steps_left_ == 0) sess_done_ = true;
    }
    const size_t take = std::min(max_tokens, sess_tokens_.size() - sess_delivered_);
    out.assign(sess_tokens_.begin() + long(sess_delivered_), sess_tokens_.begin() + long(sess_delivered_ + take));
    sess_delivered_ += take;
    if (finished) *finished = sess_done_ && sess_delivered_ == sess_tokens_.size();
    return out;
  }
  const size_t have = size_t(sess_state_.nhist) - sess_delivered_;
  if (have < max_tokens && !sess_done_) {
    const size_t steps = std::min(max_tokens - have, sess_steps_left_);
    if (steps) {
      decode_steps(int(steps));
      sess_steps_left_ -= steps;
    }
    sync_session_state();
    if (sess_steps_left_ == 0) sess_done_ = true;
  }
  const size_t avail = size_t(sess_state_.nhist) - sess_delivered_;
  const size_t take = std::min(max_tokens, avail);
  out.resize(take);
  if (take)
    check(cudaMemcpy(out.data(), hist_ + sess_delivered_, sizeof(uint32_t) * take, cudaMemcpyDeviceToHost),
          "read tokens");
  sess_delivered_ += take;
  // a KV overflow ends the loop with an error (kv_cache.rs:48-53), reported once
  // every token produced before it has been handed out
  if (take == 0 && sess_state_.err == 2)
    throw WcbError(E_PARSE, "Parse error: KV cache overflow: " + std::to_string(sess_state_.kv_len) + " + 1 > " +
                                std::to_string(max_seq_));
  if (finished) *finished = sess_done_ && sess_state_.err == 0 && sess_delivered_ == size_t(sess_state_.nhist);
  return out;
}

std::vector<uint32_t> Model::generate(const uint32_t* prompt, size_t n, const GenParams& g) {
  start(prompt, n, g);
  std::vector<uint32_t> all;
  bool fin = false;
  while (!fin) {
    std::vector<uint32_t> part = next(size_t(g.max_tokens) + 1, &fin);
    all.insert(all.end(), part.begin(), part.end());
    if (part.empty() && !fin) break;
  }
  return all;
}

}  // namespace wcb

namespace wcb {

void Model::prefill_greedy(const uint32_t* prompt, size_t n, const GenParams& g) {
  if (n > max_seq_)
    throw WcbError(E_PARSE, "Parse error: KV cache overflow: 0 + " + std::to_string(n) + " > " +
                                std::to_string(max_seq_));
  const int eos = g.eos == 0xFFFFFFFFu ? -1 : int(g.eos);
  check(launch_init_gen(st_, int(std::max<uint32_t>(g.max_tokens, 1)), eos, int(max_seq_), stream_), "init");
  check(cudaMemsetAsync(pen_cnt_, 0, sizeof(uint32_t) * cfg_.vocab, stream_), "clear penalty counts");
  rep_ = g.repetition_penalty;
  check(cudaStreamSynchronize(stream_), "prefill");  // the pinned staging buffer is free again
  std::memcpy(host_ids_, prompt, n * sizeof(uint32_t));
  check(cudaMemcpyAsync(ids_, host_ids_, n * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_), "upload ids");
  for (size_t c0 = 0; c0 < n; c0 += size_t(t_max_)) {
    const int T = int(std::min(n - c0, size_t(t_max_)));
    set_state(int(c0), int(c0), T);
    enqueue_forward(ids_ + c0, T, false);
  }
  const int last_T = int(n - ((n - 1) / size_t(t_max_)) * size_t(t_max_));
  enqueue_lm_head(last_T, true);  // samples the first token (no EOS check)
}

void Model::bind_seq(uint32_t b) {
  const size_t esz = opt_.kv_half ? 2 : 4;
  kcache_ = static_cast<uint8_t*>(kc_base_) + size_t(b) * seq_kv_elems_ * esz;
  vcache_ = static_cast<uint8_t*>(vc_base_) + size_t(b) * seq_kv_elems_ * esz;
  st_ = st_base_ + b;
  hist_ = hist_base_ + size_t(b) * hist_cap_;
  pen_cnt_ = pen_base_ + size_t(b) * cfg_.vocab;
  if (rng_base_) rng_ = rng_base_ + b;
}

int Model::batch_gemm(const DevWeight* segs, int nseg, int rows, int K, int B, const float* x, int ldx,
                      const float* norm_w, const float* sq_in, int sq_tiles, float eps, int epi, float* y, int ldy,
                      const float* resid, int ldr, float* sq_out, int layer) {
  BatchGemmArgs a{};
  for (int i = 0; i < nseg; ++i) {
    a.seg[i].w = segs[i].ptr;
    a.seg[i].dtype = segs[i].dtype;
    a.seg[i].rows = int(segs[i].rows);
  }
  a.nseg = nseg;
  a.rows = rows;
  a.K = K;
  a.B = B;
  a.x = x;
  a.ldx = ldx;
  a.norm_w = norm_w;
  a.sq_in = sq_in;
  a.sq_tiles = sq_tiles;
  a.eps = eps;
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  a.sq_out = sq_out;
  a.q = q_;
  a.ldq = int(hq_);
  if (layer >= 0) {
    const size_t esz = opt_.kv_half ? 2 : 4;
    a.kc = static_cast<uint8_t*>(kc_base_) + size_t(layer) * kv_layer_elems_ * esz;
    a.vc = static_cast<uint8_t*>(vc_base_) + size_t(layer) * kv_layer_elems_ * esz;
  }
  a.seq_stride = seq_kv_elems_;
  a.kv_half = int(opt_.kv_half);
  a.hidden = int(hq_);
  a.kv_dim = int(kvd_l_);
  a.head_dim = int(cfg_.head_dim());
  a.max_seq = int(max_seq_);
  a.rope_cos = rope_cos_;
  a.rope_sin = rope_sin_;
  a.st = st_base_;
  check(launch_batch_gemm(a, epi, stream_), "batched GEMM");
  ++batch_launches_;
  batch_gemm_plan(a, epi);
  return batch_gemm_tiles(a, epi) * a.splits;  // partial sums of squares a BEPI_RESID launch leaves
}

// One greedy decode step of slots 0..B-1 (the per-sequence semantics of the
// decode step in enqueue_forward + enqueue_lm_head): every contraction reads
// its weights once for all B sequences.
void Model::enqueue_batch_step(int B) {
  const ModelConfig& c = cfg_;
  const int H = int(c.hidden), F = int(ffn_l_), HQ = int(hq_), V = int(c.vocab);
  const int qkv_rows = HQ + 2 * int(kvd_l_);
  int sq_x = 1;  // entries of the running sums of squares of x (the embedding kernel writes one)
  batch_launches_ = 0;
  check(launch_batch_embed(emb_, V, H, st_base_, hist_base_, int(hist_cap_), x_, sqx_, B, stream_), "embed");
  ++batch_launches_;
  for (uint32_t l = 0; l < c.layers; ++l) {
    const DevLayer& L = layers_[l];
    const DevWeight qkv[3] = {L.q, L.k, L.v};
    batch_gemm(qkv, 3, qkv_rows, H, B, x_, H, L.attn_norm, sqx_, sq_x, 1e-6f, BEPI_QKV, nullptr, 0, nullptr, 0, nullptr,
               int(l));
    AttnArgs a{};
    a.q = q_;
    const size_t esz = opt_.kv_half ? 2 : 4;
    a.kc = static_cast<uint8_t*>(kc_base_) + size_t(l) * kv_layer_elems_ * esz;
    a.vc = static_cast<uint8_t*>(vc_base_) + size_t(l) * kv_layer_elems_ * esz;
    a.kv_half = int(opt_.kv_half);
    a.out = att_;
    a.part = apart_;
    a.ticket = aticket_;
    a.n_heads = int(heads_l_);
    a.n_kv = int(kv_l_);
    a.head_dim = int(c.head_dim());
    a.max_seq = int(max_seq_);
    a.T = B;
    a.chunk = BATCH_CHUNK;
    a.max_splits = asplits_;
    a.scale = attn_scale_;
    a.st = st_base_;
    a.seq_stride = seq_kv_elems_;
    check(launch_batch_attention(a, stream_), "attention");
    ++batch_launches_;
    const DevWeight o[1] = {L.o};
    const DevWeight gu[2] = {L.gate, L.up};
    const DevWeight dn[1] = {L.down};
    int sq_h;
    if (tp_ == 1) {
      sq_h = batch_gemm(o, 1, H, HQ, B, att_, HQ, nullptr, nullptr, 0, 0.0f, BEPI_RESID, h_, H, x_, H, sqh_, -1);
    } else {  // row-parallel: this rank's partial sums, all-reduced, then the residual
      batch_gemm(o, 1, H, HQ, B, att_, HQ, nullptr, nullptr, 0, 0.0f, BEPI_STORE, part_y_, H, nullptr, 0, nullptr, -1);
      all_reduce_sum(part_y_, size_t(B) * H);
      check(launch_batch_resid(h_, x_, part_y_, B, H, sqh_, stream_), "residual");
      ++batch_launches_;
      sq_h = H / BATCH_TILE;
    }
    batch_gemm(gu, 2, F, H, B, h_, H, L.ffn_norm, sqh_, sq_h, 1e-6f, BEPI_SWIGLU, act_, F, nullptr, 0, nullptr, -1);
    if (tp_ == 1) {
      sq_x = batch_gemm(dn, 1, H, F, B, act_, F, nullptr, nullptr, 0, 0.0f, BEPI_RESID, x_, H, h_, H, sqx_, -1);
    } else {
      batch_gemm(dn, 1, H, F, B, act_, F, nullptr, nullptr, 0, 0.0f, BEPI_STORE, part_y_, H, nullptr, 0, nullptr, -1);
      all_reduce_sum(part_y_, size_t(B) * H);
      check(launch_batch_resid(x_, h_, part_y_, B, H, sqx_, stream_), "residual");
      ++batch_launches_;
      sq_x = H / BATCH_TILE;
    }
  }
  const DevWeight head[1] = {lm_head_};
  const int VL = int(vocab_l_);  // this rank's LM-head rows (all of them with one rank)
  batch_gemm(head, 1, VL, H, B, x_, H, out_norm_, sqx_, sq_x, c.eps, BEPI_STORE, logits_b_, VL, nullptr, 0, nullptr,
             -1);
  if (tp_ == 1 && sample_mode_ == 1) {  // 1 <= top_k <= 1024: one sampler CTA per slot
    check(launch_sample(logits_b_, plog_, V, st_base_, hist_base_, pen_base_, rep_, samp_t_, samp_k_, samp_tp_,
                        rng_base_, stream_, B, int(hist_cap_)),
          "sampler");
    ++batch_launches_;
  } else if (tp_ == 1 && sample_mode_ == 2) {  // every other sampled configuration
    check(launch_sample_full(logits_b_, plog_, V, st_base_, hist_base_, pen_base_, rep_, samp_t_, samp_k_, samp_tp_,
                             rng_base_, nullptr, stream_, B, int(hist_cap_)),
          "sampler");
    ++batch_launches_;
  } else if (tp_ == 1) {
    check(launch_batch_sample(logits_b_, V, st_base_, hist_base_, int(hist_cap_), pen_base_, rep_, B, stream_),
          "sampler");
    ++batch_launches_;
  } else {  // vocabulary split: per-sequence keys, max all-reduced, then the bookkeeping
    check(cudaMemsetAsync(tpkeys_b_, 0, sizeof(unsigned long long) * 2 * size_t(B), stream_), "clear keys");
    check(launch_batch_keys(logits_b_, VL, int(vocab_off_), V, st_base_, pen_base_, rep_, tpkeys_b_, B, stream_),
          "argmax keys");
    const ncclResult_t r = nccl().AllReduce(tpkeys_b_, tpkeys_b_, 2 * size_t(B), ncclUint64, ncclMax, comm_, stream_);
    if (r != ncclSuccess)
      throw WcbError(E_BACKEND, std::string("Backend error: ncclAllReduce: ") + nccl().GetErrorString(r));
    check(launch_batch_finish(st_base_, tpkeys_b_, hist_base_, int(hist_cap_), pen_base_, V, B, stream_),
          "sampler bookkeeping");
    batch_launches_ += 2;
  }
}

std::vector<std::vector<uint32_t>> Model::generate_batch(const uint32_t* prompts, const size_t* lens, size_t n,
                                                         const GenParams& g) {
  check_group();
  std::vector<std::vector<uint32_t>> out(n);
  const Sampler probe(g.seed, g.temperature, g.top_p, g.top_k, g.repetition_penalty);
  // sampled configurations draw on the device (sample_dev.cu), one sampler CTA per slot
  const bool dev_sample = !probe.greedy() && plog_ && !(opt_.flags & 32);
  if (!batch_ok_ || (!probe.greedy() && !dev_sample) || n < 2) {
    size_t off = 0;
    for (size_t s = 0; s < n; ++s) {
      out[s] = generate(prompts + off, lens[s], g);
      off += lens[s];
    }
    return out;
  }
  check(cudaSetDevice(device_), "cudaSetDevice");
  sample_mode_ = dev_sample ? (probe.fixed_path(cfg_.vocab) ? 1 : 2) : 0;
  if (dev_sample) {
    samp_t_ = probe.temperature();
    samp_k_ = int(probe.top_k());
    samp_tp_ = probe.top_p();
  }
  ++session_;  // slot 0 is the single-sequence KV cache: an open session ends here
  sess_active_ = false;
  sess_done_ = true;
  kv_len_ = 0;
  std::vector<size_t> offs(n, 0);
  for (size_t s = 1; s < n; ++s) offs[s] = offs[s - 1] + lens[s - 1];
  for (size_t s = 0; s < n; ++s)
    if (lens[s] == 0) throw WcbError(E_PARSE, "Parse error: Empty token sequence");
  std::vector<StepState> hs(bslots_);
  for (size_t g0 = 0; g0 < n; g0 += bslots_) {
    const int B = int(std::min<size_t>(bslots_, n - g0));
    if (dev_sample) {  // each sequence draws from the seed's stream, as its own generate() does
      const std::vector<StdRng> seeds(size_t(B), probe.seed_state());
      check(cudaMemcpyAsync(rng_base_, seeds.data(), sizeof(StdRng) * seeds.size(),
                            cudaMemcpyHostToDevice, stream_),
            "seed");
      check(cudaStreamSynchronize(stream_), "seed");
    }
    try {
      for (int b = 0; b < B; ++b) {
        bind_seq(uint32_t(b));
        prefill_greedy(prompts + offs[g0 + b], lens[g0 + b], g);
      }
    } catch (...) {
      bind_seq(0);
      throw;
    }
    bind_seq(0);
    const bool same_sampler = batch_graph_mode_ == sample_mode_ &&
                              (sample_mode_ == 0 || (batch_graph_t_ == samp_t_ && batch_graph_k_ == samp_k_ &&
                                                     batch_graph_tp_ == samp_tp_));
    if (!batch_exec_ || batch_graph_b_ != B || batch_graph_rep_ != rep_ || !same_sampler) {
      if (batch_exec_) {
        cudaGraphExecDestroy(batch_exec_);
        cudaGraphDestroy(batch_graph_);
        batch_exec_ = nullptr;
        batch_graph_ = nullptr;
      }
      cudaGraph_t gr = nullptr;
      check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
      try {
        enqueue_batch_step(B);
      } catch (...) {
        cudaStreamEndCapture(stream_, &gr);
        if (gr) cudaGraphDestroy(gr);
        throw;
      }
      check(cudaStreamEndCapture(stream_, &gr), "end capture");
      cudaGraphExec_t e = nullptr;
      const cudaError_t r = cudaGraphInstantiate(&e, gr, 0);
      if (r != cudaSuccess) {
        cudaGraphDestroy(gr);
        check(r, "graph instantiate");
      }
      batch_graph_ = gr;
      batch_exec_ = e;
      batch_graph_b_ = B;
      batch_graph_rep_ = rep_;
      batch_graph_mode_ = sample_mode_;
      batch_graph_t_ = samp_t_;
      batch_graph_k_ = samp_k_;
      batch_graph_tp_ = samp_tp_;
    }
    // decode steps for the whole group; finished sequences are skipped by the
    // sampler and their KV caches are no longer written
    size_t steps_left = g.max_tokens > 1 ? size_t(g.max_tokens) - 1 : 0;
    auto read_states = [&]() {
      check(cudaMemcpyAsync(hs.data(), st_base_, sizeof(StepState) * size_t(B), cudaMemcpyDeviceToHost, stream_),
            "read states");
      check(cudaStreamSynchronize(stream_), "batched decode");
      for (int b = 0; b < B; ++b) {
        if (hs[b].err & 28)
          throw WcbError(E_BACKEND, "Backend error: batched decode: a bounded wait expired (device error word " +
                                        std::to_string(hs[b].err) + ")");
        if (hs[b].err & 1) throw WcbError(E_GENERIC, "Runtime error: NaN logit");
      }
    };
    read_states();
    auto all_done = [&]() {
      for (int b = 0; b < B; ++b)
        if (!hs[b].done) return false;
      return true;
    };
    while (steps_left > 0 && !all_done()) {
      const size_t k = std::min<size_t>(steps_left, 16);
      for (size_t i = 0; i < k; ++i) check(cudaGraphLaunch(batch_exec_, stream_), "graph launch");
      steps_left -= k;
      read_states();
    }
    for (int b = 0; b < B; ++b) {
      if (hs[b].err == 2)  // the KV append of a further step would overflow (kv_cache.rs:48-53)
        throw WcbError(E_PARSE, "Parse error: KV cache overflow: " + std::to_string(hs[b].kv_len) + " + 1 > " +
                                    std::to_string(max_seq_));
      std::vector<uint32_t>& o = out[g0 + size_t(b)];
      o.resize(size_t(hs[b].nhist));
      if (!o.empty())
        check(cudaMemcpy(o.data(), hist_base_ + size_t(b) * hist_cap_, sizeof(uint32_t) * o.size(),
                         cudaMemcpyDeviceToHost),
              "read tokens");
    }
  }
  return out;
}

}  // namespace wcb
