// Device kernels of the token loop and their host launchers.
//
// HBM layout (one model replica):
//   weights   raw GGUF blocks, row-major [rows][K/256 blocks]: Q4_K 144 B/block,
//             Q6_K padded to 224 B/block (first 210 bytes unchanged)
//   embedding f32 [vocab][hidden] (token_embd as stored in the GGUF)
//   KV cache  per layer: K and V, [n_kv_heads][max_seq][head_dim], f32 or f16
//   RoPE      cos/sin tables [max_seq][head_dim/2] computed on the host with the
//             reference formula (attention.rs:230-248), so rotations are bit-exact
//   StepState one small struct the kernels read position / KV length from, so a
//             decode step can be captured once in a CUDA graph and replayed
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace wcb {

struct StdRng;  // the sampled draws' random stream (sample_int.h)

constexpr int QK_K = 256;
constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;
constexpr int Q6K_DEV_BYTES = 224;
constexpr int DT_F32 = 0;   // dense weights (GGUF types 0 / 1): per-op kernels only
constexpr int DT_F16 = 1;
constexpr int DT_Q4K = 12;
constexpr int DT_Q6K = 14;

#ifdef __CUDACC__
#define WCB_HD __host__ __device__
#else
#define WCB_HD
#endif
// bytes of 256 consecutive values of a row in device memory
WCB_HD inline size_t dev_block_bytes(int dtype) {
  return dtype == DT_Q4K ? Q4K_BYTES : dtype == DT_Q6K ? Q6K_DEV_BYTES : dtype == DT_F32 ? 1024 : 512;
}
WCB_HD inline bool dense_dtype(int dtype) { return dtype == DT_F32 || dtype == DT_F16; }

// State shared by the kernels of one forward / decode step (device memory).
struct StepState {
  unsigned long long best;  // LM-head argmax key: (order-preserving logit bits << 32) | index
  int position;  // RoPE position / causal-mask base of token 0 of this forward
  int kv_len;    // KV length before this forward (slot of token 0)
  int n_tokens;  // tokens in this forward
  int done;      // decode loop finished: kernels of later steps return at once
  int gen;       // tokens generated so far (generate loop)
  int max_gen;   // generate's max_tokens
  int nhist;     // sampler history length (LogitsProcessor::previous_tokens)
  int err;       // device error word: 1 = NaN logit (sampler), 2 = KV overflow
  int eos;       // EOS id (-1: none)
  int max_seq;   // KV capacity
  int ticket;    // LM-head CTAs finished (the last one runs the sampler bookkeeping)
  int nan;       // a penalised logit was NaN
  int epoch;     // persistent decode step: launches so far (tags of this launch's activations)
  int wait_ms;   // bound of the device-side waits on other ranks / CTAs (0: 2000 ms)
};
static_assert(sizeof(StepState) == 64, "StepState layout");

// ---------------------------------------------------------------- GEMV ----
enum GemvPro { PRO_NONE = 0, PRO_RMSNORM = 1 };
// EPI_LMHEAD: store the logits and, in generate mode, fuse the repetition
// penalty, the argmax and generate()'s bookkeeping (sampling.rs:86-125,
// model.rs:1380-1409) into the LM-head launch.
// EPI_PEER (tensor parallelism, one token): each output is a partial sum; it is
// written as a (value, tag) pair into slot `tp_rank` of every rank's receive
// buffer over NVLink, and launch_tp_reduce_add sums the slots on each rank.
enum GemvEpi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_LMHEAD = 4, EPI_PEER = 5 };

struct GemvSeg {
  const uint8_t* w;
  int dtype;
  int rows;
};

struct GemvArgs {
  GemvSeg seg[3];
  int nseg;
  int K;
  int M;              // activation rows (tokens) in this launch
  int ngroups;        // row groups of 4
  int ksplit;         // K slices per row group (set by launch_gemv)
  int stage_groups;   // row groups per shared-memory stage (set by launch_gemv)
  int slot_bytes;     // bytes of one stage slot (set by launch_gemv)
  const float* x;     // [M][ldx] input (PRO_NONE) or residual stream h (PRO_RMSNORM)
  int ldx;
  const float* norm_w;  // PRO_RMSNORM weight
  float eps;
  float* y;           // EPI_STORE / EPI_RESID / EPI_SWIGLU output [M][ldy]
  int ldy;
  const float* resid;  // EPI_RESID residual [M][ldr]
  int ldr;
  // EPI_QKV
  float* q;           // [M][ldq]
  int ldq;
  void* kc;           // this layer's K cache [n_kv][max_seq][hd]
  void* vc;
  int kv_half;        // KV element type: 0 f32, 1 f16
  int hidden;
  int kv_dim;
  int head_dim;
  int max_seq;
  const float* rope_cos;  // [max_seq][head_dim/2]
  const float* rope_sin;
  StepState* st;
  int token_offset;   // first token of this launch within the forward (column groups)
  int row_offset;     // EPI_QKV: first q/k/v row of this launch
  // EPI_LMHEAD
  int gen_mode;            // 1: penalty + argmax + generate bookkeeping; 2: penalty + argmax key only
  int vocab_off;           // token id of LM-head row 0 (tensor parallelism: this rank's first row)
  const uint32_t* pen_cnt; // occurrences of each token in the sampler history
  uint32_t* pen_cnt_w;     // same array, incremented when a token is pushed
  float rep;               // repetition penalty
  uint32_t* hist;          // sampler history
  // EPI_PEER
  unsigned long long* const* peers;  // [tp_size] receive buffers [tp_size][ldy] (device array of pointers)
  int tp_rank, tp_size;
  int peer_phase;                    // tag of these partials: epoch * 512 + peer_phase + 1
  // 1: launch with programmatic dependent launch. Only for static weights: the
  // kernel reads its weights before waiting on the previous kernel.
  int pdl;
  // tensor-core GEMM: the activations prepared by launch_stage_x (null: staged in the kernel)
  const uint8_t* xprep;
};

// shared memory of the activation planes of M columns of K values (+ a
// 8 x 16 float reduction scratch)
WCB_HD inline size_t gemv_planes_bytes(int M, int K) {
  return size_t(3) * M * K + sizeof(float) * 2 * size_t(M) * (K / 32) + sizeof(float) * 8 * 16;
}
int gemv_max_cols(int K);  // widest column group whose activation planes fit in shared memory
cudaError_t launch_gemv(const GemvArgs& a, int pro, int epi, cudaStream_t s);

// Tensor-core (tcgen05) GEMM for prefill: same arguments and epilogues as the
// GEMV (EPI_STORE, EPI_RESID, EPI_QKV, EPI_SWIGLU), a.M = tokens (any count),
// row_m = per-token RMSNorm divisors from launch_row_rms when pro == PRO_RMSNORM.
cudaError_t gemm_tc_configure();
cudaError_t launch_gemm_tc(const GemvArgs& a, int pro, int epi, const float* row_m, cudaStream_t s);
cudaError_t launch_row_rms(const float* x, int ldx, int T, int K, float eps, float* m, bool pdl, cudaStream_t s);
// the A tiles of launch_gemm_tc (fp16 hi / lo, times norm_w when not null) into out,
// stage_x_bytes(T, K) bytes
cudaError_t launch_stage_x(const float* x, int ldx, int T, int K, const float* norm_w, uint8_t* out, cudaStream_t s);
size_t stage_x_bytes(int T, int K);
constexpr int TC_MIN_TOKENS = 16;  // below this the GEMV (dp4a) path is used

// ----------------------------------------------------------- attention ----
struct AttnArgs {
  const float* q;     // [T][n_heads][hd] (post-RoPE)
  const void* kc;     // [n_kv][max_seq][hd]
  const void* vc;
  int kv_half;
  float* out;         // [T][n_heads][hd]
  float* part;        // scratch: [T][n_heads][max_splits][hd + 2]
  int* ticket;        // scratch: [T][n_kv], zero between launches
  int n_heads, n_kv, head_dim, max_seq;
  int T;
  int chunk;          // keys per split
  int max_splits;
  float scale;        // 1 / sqrt(head_dim)
  const StepState* st;
  // launch_batch_attention: "token" t is sequence t with one query at
  // st[t].position over its own cache (kc / vc + t * seq_stride elements)
  size_t seq_stride;
};
constexpr int ATT_TILE = 32;  // keys staged in shared memory per pass
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s);
// Prefill attention on the tensor cores (mma.sync, fp16 hi/lo operands, fp32
// accumulate): the T query tokens of a forward chunk (a.chunk / a.max_splits /
// a.part / a.ticket unused). Head dims 64 / 128, n_heads / n_kv in {1, 2, 4, 8}.
cudaError_t attention_prefill_configure();
bool attention_prefill_supported(int n_heads, int n_kv, int head_dim);
cudaError_t launch_attention_prefill(const AttnArgs& a, cudaStream_t s);

// ------------------------------------------------ persistent decode step --
// One launch runs a whole decode step (T = 1): every layer's QKV + RoPE + KV
// append, attention, output projection + residual, gate/up + SwiGLU, down +
// residual, then the final norm, LM head and, in generate mode, penalty,
// argmax and generate()'s bookkeeping. One CTA per SM (cooperative launch,
// so all CTAs are resident). Each CTA owns a fixed share of every weight
// matrix; its weight tiles stream through a ring of shared-memory slots with
// bulk copies that run ahead across phases (weights do not depend on the
// activations). Activations that cross CTAs are (value, tag) pairs written
// with one 64-bit store: a consumer spins on the elements it reads until they
// carry the tag of the producing phase of this step, so no counters, fences
// or grid barriers sit between phases.
enum MkKind { MK_QKV = 0, MK_ATT = 1, MK_O = 2, MK_GU = 3, MK_D = 4, MK_LM = 5 };

// One weight "part" of a phase: rows of one quantisation type, processed in
// groups of 4 rows (MK_GU: 2 gate + 2 up rows, giving 2 outputs). 64 bytes:
// a launch keeps the whole list in shared memory. Phases are numbered 5 per
// layer (QKV, attention, o, gate/up, down) and then the LM head, so a part's
// layer is phase / 5.
struct MkPart {
  const uint8_t* w[3];  // MK_QKV: segments of the virtual [q; k; v] matrix; MK_GU: gate, up; else w[0]
  const float* norm;    // RMSNorm weight of the phase input (null: none)
  int rows0, rows1;     // rows of segments 0 and 1 (segment 2 holds the rest)
  int K;                // input length
  uint16_t ngroups;     // 4-row groups (gate / up: 2 gate + 2 up rows)
  uint16_t gpt;         // groups of one weight tile (set by decode_step_plan)
  int row_offset;       // MK_QKV: row of the virtual matrix at this part's row 0
  float eps;
  int16_t phase;        // phase index (tags of its outputs)
  int16_t dep;          // phase whose outputs this phase reads (-1: the embedding row)
  uint8_t kind;         // MkKind
  uint8_t first;        // first part of its phase (builds the input planes)
  uint8_t dtype;        // DT_Q4K / DT_Q6K (MK_ATT: unused)
  uint8_t nseg;
  // K chain (a down projection whose input is longer than MK_MAX_INPUT): the part
  // covers input values [kofs, kofs + K) of rows row_stride bytes apart; its 8-block
  // chunks are chunks kch0.. of the kchs of the whole row. kchain 1: more parts of the
  // chain follow (their partial sums accumulate, no epilogue); 2: the last part.
  int kofs;
  int row_stride;       // bytes between weight rows (0: rows of K values are contiguous)
  int16_t kch0, kchs;
  uint8_t kchain;
  uint8_t pad[3];
};
static_assert(sizeof(MkPart) == 80, "MkPart layout");
constexpr int MK_MAX_INPUT = 16384;  // longest input of one part of the persistent decode step

// A tile: ng groups starting at group g of part `part` (whole K rows).
struct MkTile {
  uint16_t g;
  uint16_t part;
  uint8_t ng;
};

struct MkArgs {
  const MkPart* parts;
  int nparts;
  StepState* st;
  const float* emb;
  int vocab, hidden, ffn, n_heads, n_kv, head_dim, max_seq;
  const float* rope_cos;
  const float* rope_sin;
  void* kcache;  // [layers][n_kv][max_seq][hd]
  void* vcache;
  size_t kv_layer_elems;
  int kv_half;
  float attn_scale;
  // tagged activations: (float bits, tag) in one 64-bit word
  unsigned long long* xa;    // residual stream between layers [hidden]
  unsigned long long* xb;    // residual stream after attention [hidden]
  unsigned long long* q;     // post-RoPE queries [hidden]
  unsigned long long* knew;  // this step's K / V rows [n_kv * head_dim]
  unsigned long long* vnew;
  unsigned long long* att;   // attention output [att_smax][hidden]: key split s's normalised partial
  unsigned long long* attml; // [att_smax][n_heads][2] each split's softmax max and sum (splits > 1)
  unsigned long long* act;   // SwiGLU output [ffn]
  float* logits;             // [vocab]
  const float* zero;         // [hidden] zeros: the embedding of an out-of-vocabulary id
  int att_smax;              // most key splits of a query head (set by decode_step_plan)
  int has_q6;                // a weight of the step is Q6_K (set by decode_step_plan)
  // tests of the bounded waits: the outputs of this phase are never written, so the
  // waits of its consumers run out (wait_ms) and the launch ends with an error (-1: none)
  int drop_phase;
  int gen_mode;              // 1: token = hist[nhist - 1], penalty + argmax + bookkeeping;
                             // 2: token = hist[nhist - 1], logits only (a sampler kernel follows)
  const uint32_t* ids;       // gen_mode 0: token = ids[0]
  uint32_t* hist;
  uint32_t* pen_cnt;
  float rep;
  // tensor parallelism (tp_size > 1): this rank holds its shard (heads, FFN rows and
  // vocabulary rows); the o / down partial sums and the LM-head argmax keys reach
  // every rank by peer stores into its exchange buffer, whose decode-step region is
  // [o, down][layer parity][rank][hidden] tagged words, then [rank][2] key words
  int tp_size, tp_rank;
  int qdim;                          // query rows of the [q; k; v] part (hidden with one rank)
  int vocab_off;                     // token id of this rank's first LM-head row
  unsigned long long* const* peers;  // [tp_size] every rank's exchange buffer
  size_t xofs;                       // offset (words) of the decode step's region in each buffer
  // shared-memory layout (from decode_step_plan)
  int slot_bytes, nslots, region_bytes, kmax;
  int part_floats;  // partial sums of a split part's chunks (longest share x chunks x 4)
  int res_rows;   // rows of an O / D share
  int lm_rows;    // LM-head rows a CTA owns
};
// Sets each part's tile size (gpt) and the shared-memory layout; false when the
// model does not fit the persistent kernel (then the per-op kernels run).
bool decode_step_plan(MkPart* parts, int nparts, MkArgs& a, int n_rep, size_t* smem);
int decode_step_grid();  // CTAs of one launch (one per SM)
cudaError_t decode_step_configure();
cudaError_t launch_decode_step(const MkArgs& a, size_t smem, cudaStream_t s);

// ------------------------------------------------ batched decode (serving) --
// One greedy decode step of B independent sequences (generate_batch): the
// weight contractions run on the tensor cores (tcgen05.mma, kind::f16) with the
// 128 weight rows of a tile as the MMA M dimension and the B sequences as N.
// The 4- / 6-bit quants are integers, exact in fp16, so the A operand is the
// raw quant and the B operand the activation split into fp16 hi + lo halves;
// each Q4_K sub-block (32 values) / Q6_K sub-block (16) accumulates into its
// own TMEM columns and the CUDA cores apply y += d*sc * dot - dmin*m * sum(x).
// K is split over the CTAs of one thread-block cluster per tile; the slices are
// added in slice order over distributed shared memory (deterministic) and the
// cluster's CTAs share the fused epilogue.
enum BatchEpi { BEPI_STORE = 0, BEPI_RESID = 1, BEPI_SWIGLU = 2, BEPI_QKV = 3 };
constexpr int BATCH_MAX = 32;   // sequences of one batched step (MMA N <= 32)
constexpr int BATCH_TILE = 128; // weight rows of one tile (BEPI_SWIGLU: 64 gate + 64 up rows)

struct BatchGemmArgs {
  GemvSeg seg[3];        // rows of the virtual matrix: seg 0, then 1, then 2 (BEPI_SWIGLU: gate, up)
  int nseg;
  int rows;              // virtual rows (BEPI_SWIGLU: gate rows = up rows = outputs)
  int K;                 // input length, a multiple of 256
  int B;                 // sequences (1..BATCH_MAX)
  const float* x;        // [B][ldx]
  int ldx;
  const float* norm_w;   // RMSNorm weight of the input (null: no norm)
  const float* sq_in;    // [sq_tiles][B] partial sums of squares of x (summed in order)
  int sq_tiles;
  float eps;
  int splits;            // K slices = CTAs of a tile's cluster (set by batch_gemm_plan, <= 8)
  int sb_per_split;      // super-blocks per slice (set by batch_gemm_plan)
  float* y;              // BEPI_STORE / RESID / SWIGLU output [B][ldy]
  int ldy;
  const float* resid;    // BEPI_RESID [B][ldr]
  int ldr;
  float* sq_out;         // BEPI_RESID: [tiles * splits][B] sums of squares of each CTA's outputs
  // BEPI_QKV: RoPE'd queries to q, RoPE'd keys and values appended to each sequence's cache
  float* q;
  int ldq;
  void* kc;              // this layer's caches of sequence 0 [n_kv][max_seq][hd]
  void* vc;
  size_t seq_stride;     // elements from one sequence's cache to the next
  int kv_half, hidden, kv_dim, head_dim, max_seq;
  const float* rope_cos;
  const float* rope_sin;
  StepState* st;         // [B]
};
// tiles and slices of a launch (CTAs = tiles * splits; a BEPI_RESID launch
// writes tiles * splits partial sums of squares per sequence)
int batch_gemm_tiles(const BatchGemmArgs& a, int epi);
void batch_gemm_plan(BatchGemmArgs& a, int epi);
cudaError_t batch_configure();
cudaError_t launch_batch_gemm(BatchGemmArgs a, int epi, cudaStream_t s);
// Decode attention of B sequences (one query each, n_heads / n_kv <= 8): grid
// (n_kv, B, max_splits), a.chunk keys per split, merged by the last CTA of a
// (sequence, kv head); K rows and V rows are read straight from the cache
cudaError_t launch_batch_attention(const AttnArgs& a, cudaStream_t s);
// tensor parallelism: y[b] = resid[b] + add[b] (the all-reduced partial sums) with
// per-128-row-tile sums of squares sq[tile][b]; the vocabulary-split LM head's
// per-sequence keys (keys[2b] = best (logit bits << 32 | id), keys[2b+1] = NaN seen,
// zeroed before, max all-reduced after) and the bookkeeping from the reduced keys
cudaError_t launch_batch_resid(float* y, const float* resid, const float* add, int B, int H, float* sq,
                               cudaStream_t s);
cudaError_t launch_batch_keys(const float* logits, int vl, int vocab_off, int vocab, const StepState* st,
                              const uint32_t* pen_cnt, float rep, unsigned long long* keys, int B, cudaStream_t s);
cudaError_t launch_batch_finish(StepState* st, const unsigned long long* keys, uint32_t* hist, int hist_cap,
                                uint32_t* pen_cnt, int vocab, int B, cudaStream_t s);
// x[b] = embedding row of sequence b's last token; sq[b] = sum of squares of x[b]
cudaError_t launch_batch_embed(const float* emb, int vocab, int hidden, const StepState* st, const uint32_t* hist,
                               int hist_cap, float* x, float* sq, int B, cudaStream_t s);
// per sequence: repetition penalty, argmax (last maximum wins) and generate()'s
// bookkeeping into st[b], hist + b * hist_cap, pen_cnt + b * vocab
cudaError_t launch_batch_sample(const float* logits, int vocab, StepState* st, uint32_t* hist, int hist_cap,
                                uint32_t* pen_cnt, float rep, int B, cudaStream_t s);

// ------------------------------------------------------------ sampling ----
// Temperature + top-k (+ top-p) draw on the device for one sequence (1 <= top_k
// <= 1024): penalty into `scratch` [n], the draw with the random stream *rng
// (the host Sampler's fixed-order path, operation for operation), then
// generate()'s bookkeeping on st / hist / pen_cnt
// nseq > 1: one CTA per sequence b of a batch, over logits / scratch / pen_cnt + b * n,
// st + b, hist + b * hist_stride and rng + b (the batched decode step).
cudaError_t launch_sample(const float* logits, float* scratch, int n, StepState* st, uint32_t* hist,
                          uint32_t* pen_cnt, float rep, float temperature, int top_k, float top_p,
                          StdRng* rng, cudaStream_t s, int nseq = 1, int hist_stride = 0);
// The same draw for every other sampled configuration (top_k = 0: all tokens, or
// top_k > 1024), over integer weights (sample_int.h) so that the host sampler's
// Sampler::sample_int keeps the same candidates and draws the same token; probs
// (device, may be null) receives each token's final probability.
cudaError_t launch_sample_full(const float* logits, float* scratch, int n, StepState* st, uint32_t* hist,
                               uint32_t* pen_cnt, float rep, float temperature, int top_k, float top_p,
                               StdRng* rng, float* probs, cudaStream_t s, int nseq = 1,
                               int hist_stride = 0);

// ------------------------------------------------------------ elementwise --
cudaError_t launch_embed(const float* emb, int vocab, int hidden, const uint32_t* ids, int T, float* x,
                         const StepState* st, cudaStream_t s);
// decode-step embedding: id = hist[nhist - 1]
cudaError_t launch_embed_last(const float* emb, int vocab, int hidden, const uint32_t* hist, float* x,
                              const StepState* st, cudaStream_t s);

// dst = a + b elementwise (the residual add after a tensor-parallel all-reduce)
cudaError_t launch_add(float* dst, const float* a, const float* b, size_t n, const StepState* st, cudaStream_t s);
// tensor-parallel LM head: st->best / st->nan -> key[0..1] before a max
// all-reduce over the ranks, then the reduced key back and generate()'s bookkeeping
cudaError_t launch_tp_pack_key(StepState* st, unsigned long long* key, cudaStream_t s);
// dst[i] = resid[i] + sum over ranks r (in rank order) of recv[r * n + i], each
// value waited for (bounded) until it carries the tag epoch * 512 + phase + 1;
// an expired wait sets st->err bit 16
cudaError_t launch_tp_reduce_add(float* dst, const float* resid, const unsigned long long* recv, int tp_size,
                                 size_t n, int phase, StepState* st, cudaStream_t s);
cudaError_t launch_tp_finish(StepState* st, const unsigned long long* key, uint32_t* hist, uint32_t* pen_cnt,
                             cudaStream_t s);
// the same reduction of the LM-head keys without NCCL: this rank's key goes as two
// tagged 64-bit words (tag epoch * 512 + 512: the high and low key words, the NaN
// flag in bit 31 of the low one) into slot tp_rank of every rank's receive buffer
// at key_off; then a bounded wait for every rank's pair, the maximum key, the
// bookkeeping. An expired wait sets st->err bit 16 and ends the step (st->done).
cudaError_t launch_tp_key_exchange(StepState* st, unsigned long long* const* peers, const unsigned long long* own,
                                   int tp_rank, int tp_size, size_t key_off, uint32_t* hist, uint32_t* pen_cnt,
                                   cudaStream_t s);

// StepState writers (single-thread kernels, so they order with the stream and
// can sit inside a captured graph)
cudaError_t launch_set_state(StepState* st, int position, int kv_len, int n_tokens, cudaStream_t s);
cudaError_t launch_init_gen(StepState* st, int max_gen, int eos, int max_seq, cudaStream_t s);
// kernels launched with programmatic dependent launch (PDL): a kernel may start
// while its predecessor drains, prefetching weights before it waits on it
void set_pdl(bool on);
// sets the shared-memory limits of every GEMV instantiation (before any capture)
cudaError_t gemv_configure_all();

cudaError_t launch_dequant(const void* blocks, int dtype, size_t nblocks, float* out, cudaStream_t s);
cudaError_t launch_repack_q6k(const void* packed, size_t nblocks, void* padded, cudaStream_t s);

}  // namespace wcb
