// Shapes, the per-session control block and kernel argument blocks shared by
// host and device code. The model shape is the one source/src/model.rs:7-9,
// :41-78 hard-codes (hidden 1024, 24 layers with layer l%4==3 full attention,
// MLP 3584, vocab 248,320, GDN 16 heads x 128, attention 8 q / 2 kv heads x 256).
#pragma once
#include <cuda.h>  // CUtensorMap (TMA descriptors in the GEMM arguments)
#include <stdint.h>

namespace q35 {

constexpr int kHidden = 1024;
constexpr int kLayers = 24;
constexpr int kMlp = 3584;
constexpr int kVocab = 248320;
constexpr int kGdnHeads = 16;
constexpr int kGdnDim = 128;
constexpr int kGdnConv = 6144;  // q 2048 | k 2048 | v 2048
constexpr int kQHeads = 8;
constexpr int kKvHeads = 2;
constexpr int kHeadDim = 256;
constexpr int kQProj = 4096;  // per q head: query 256 | gate 256
constexpr uint32_t kDefaultCapacity = 262144;  // model.rs:8

// Attention geometry: one CTA per (chain, kv head); a chain is the
// reference's block of keys b, b + stride, ... (stride 32 below 1024 keys,
// 64 from 1024 on).
constexpr int kAttnChains = 64;
constexpr int kAttnTile = 32;   // keys of one chain per ring stage
constexpr int kAttnStages = 4;   // K and V ring depth (tiles)
constexpr int kAttnThreads = 576; // 8 score, 4 scan, 4 recurrence, 2 producer warps
constexpr int kAttnBufs = 4;      // score and f/e hand-off buffers between warp roles

// Head (vocabulary projection + greedy) geometry.
constexpr int kHeadThreads = 384;                      // 12 warps, 4 rows each per chunk
constexpr int kHeadRowsPerChunk = 4 * kHeadThreads / 32;  // 48
constexpr int kHeadChunksPerCta = 35;
constexpr int kHeadRowsPerCta = kHeadRowsPerChunk * kHeadChunksPerCta;  // 1680
constexpr int kHeadCtas = (kVocab + kHeadRowsPerCta - 1) / kHeadRowsPerCta;  // 148
constexpr int kHeadStages = 4;
constexpr int kPrefillTokens = 16;  // prompt tokens per chunk launch
// graph launches (prompt chunks) the token loop keeps queued: with 8 decode
// steps per graph at most 16 steps are in flight when a cancel arrives, as
// the reference's bounded-ahead loop keeps (model.rs:127)
constexpr int kInflight = 2;

// Device-resident control block of one decode session (or one op call).
struct Ctl {
  uint32_t pos;        // next position to consume (host sets it; advanced on device)
  uint32_t pos_step;   // position consumed by the running step
  uint32_t out_count;  // tokens emitted by the running request
  uint32_t err;        // nonzero: a bounded wait expired (value = site code)
  uint32_t head_counter;
  uint32_t attn_counter[kKvHeads];
  uint32_t capacity;
  float rope_cs[64];   // cos/sin of the running step's position, pairs i<32
  uint32_t token_step; // token consumed by the running step
  // in-kernel timing of the attention launches (device clock, ns)
  uint32_t timing_on;
  uint32_t attn_done;            // CTAs finished in the running launch
  uint32_t attn_launches;        // launches accounted
  unsigned long long attn_t0;    // earliest post-dependency start of the running launch
  unsigned long long attn_ns;    // summed launch durations
  uint32_t epoch;      // reset generation (sequence-split exchange tags)
  // in-kernel timing of the matvec launches (same switch, same clock)
  uint32_t qmv_done;             // CTAs finished in the running launch
  uint32_t qmv_launches;         // launches accounted
  unsigned long long qmv_t0;     // earliest post-dependency start of the running launch
  unsigned long long qmv_ns;     // summed launch durations
  unsigned long long qmv_bytes;  // summed algorithmic bytes (codes, scales, biases)
  unsigned long long attn_tend;  // latest CTA end of the running attention launch
  unsigned long long qmv_tend;   // latest CTA end of the running matvec launch
};

// Error site codes written to Ctl::err.
enum : uint32_t {
  kErrQmvWait = 1,
  kErrAttnWait = 2,
  kErrHeadWait = 3,
  kErrRecurWait = 4,
  kErrToken = 5,
  kErrProbeWait = 6,  // the diagnostic bounded-wait probe
  kErrXWait = 7,      // sequence split: a peer's attention record did not arrive
};

// ---- Q4 matvec kernel arguments ----
enum : int { kProPlain = 0, kProRms = 1, kProEmbedRms = 2, kProNormGate = 3 };
enum : int { kEpiStore = 0, kEpiResAdd = 1, kEpiSwiglu = 2, kEpiGdnConv = 3 };

struct QmvSeg {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  uint16_t* y;
  int rows;
};

struct QmvArgs {
  QmvSeg seg[4];
  int nseg;
  int K;
  int units;          // rows, or activation rows for SwiGLU
  int units_per_cta;
  int pro, epi;
  const uint16_t* x;     // plain / RMS input
  const uint16_t* gain;  // RMS gain
  uint16_t* h_out;       // embedding prologue: residual stream (written by CTA 0)
  const uint32_t* ew;    // embedding matrix (Q4)
  const uint16_t* es;
  const uint16_t* eb;
  const uint32_t* seq;   // token ring [capacity + 1]
  const uint16_t* gy;    // norm-gate prologue: recurrence output [2048]
  const uint16_t* gz;    // z projection [2048]
  const uint16_t* gw;    // norm weight [128]
  const float* gzs;      // norm-gate prologue: precomputed z * sigmoid(z) [rows][2048] (optional)
  float* zs_out;         // GDN input projection: z * sigmoid(z) of the z rows, f32 [2048] (optional)
  uint16_t* res;         // residual (in/out) for kEpiResAdd
  uint16_t* hist;        // GDN conv history [3][6144]
  const uint16_t* convw; // [6144][4]
  uint16_t* conv_out;    // [6144]
  Ctl* ctl;
  int advance_pos;       // this launch moves ctl->pos to pos_step + 1
  // prompt chunks (k_qmv_chunk only): ntok consecutive tokens, `sub` of them
  // in shared memory at a time; token t's rows of x / gy / gz / res /
  // conv_out and of seg[s].y sit at t * (row width) (ystride[s] for seg[s].y)
  int ntok, sub;
  int ystride[4];
  float* rope_out;       // embedding prologue: [ntok][64] RoPE table of the chunk
  // batched sessions (sess != 0): token t is the pending token of session t,
  // whose control block, token ring and conv history come from these device
  // tables (history of this layer at hists[t] + hist_off)
  int sess;
  Ctl* const* ctls;
  uint32_t* const* seqs;
  uint16_t* const* hists;
  size_t hist_off;
};

struct RecurArgs {
  const uint16_t* conv;   // [6144] post-SiLU conv output (q,k not yet normalised)
  const uint16_t* a_raw;  // [16]
  const uint16_t* b_raw;  // [16]
  const float* a_log;     // [16]
  const uint16_t* dt_bias;// [16]
  float* state;           // [16][128 v][128 k]
  uint16_t* y;            // [2048]
  Ctl* ctl;
  int advance_pos;
  int ntok;               // prompt chunks: conv [ntok][6144], a/b [ntok][32], y [ntok][2048]
  // batched sessions: session z's state at states[z] + state_off, control block ctls[z]
  float* const* states;
  size_t state_off;
  Ctl* const* ctls;
  // optional: the output gate z * sigmoid(z) in f32 (gdn.metal:246-253), formed
  // once per channel from z [rows][2048] for the norm-gate prologue
  const uint16_t* z;
  float* zs;
};

struct AttnArgs {
  const uint16_t* q_raw;  // [8][512] query | gate per head
  const uint16_t* k_raw;  // [2][256]
  const uint16_t* v_raw;  // [2][256]
  const uint16_t* q_gain; // [256]
  const uint16_t* k_gain; // [256]
  uint16_t* kcache;       // [2][64 chains][capacity/64][256], position p at chain p%64, slot p/64
  uint16_t* vcache;
  uint32_t capacity;
  float* part_o;          // [2][kAttnChains][4][256]
  float* part_ml;         // [2][kAttnChains][4][2]
  uint16_t* gated;        // [8][256]
  Ctl* ctl;
  int pos_add;            // prompt chunks: this token sits at ctl->pos_step + pos_add
  const float* rope;      // prompt chunks: its RoPE table [64] (else ctl->rope_cs)
  // Sequence split over xworld ranks (xworld <= 1: off). This rank keeps the
  // K/V of positions p with p % xworld == xrank at local index p / xworld
  // (capacity is then the local capacity); the combine exchanges per-rank
  // (m, l, o) records through every rank's receive buffer (xrecv, xflag:
  // device addresses of each rank's buffers, this rank's included).
  int xrank, xworld, xlayer;
  uint32_t xwait_ms;  // bound of the wait for the peers' records (0: 10 s)
  float* const* xrecv;
  unsigned long long* const* xflag;
  // batched sessions (launch grid z = session): each session's cache and
  // control block; its q/k/v, gated, RoPE and partial rows sit at z times the
  // row size from the pointers above
  const struct AttnSess* sess;
  float nzero;  // -0.0f, set by launch_attn*: the run-time addend of the packed products (prod2)
};

struct AttnSess {
  uint16_t* kcache;
  uint16_t* vcache;
  Ctl* ctl;
  uint32_t capacity;
};

// Q4 affine GEMM on the tensor cores (several tokens per launch):
// y[t][n] = bf16(sum_k W[n][k] x[t][k]) (+ residual), W = bf16(s q + b), for
// up to kGemmSegs weight matrices sharing the input x (a fused row space).
constexpr int kGemmSegs = 4;
struct QGemmSeg {
  const uint32_t* w;     // [rows][K/8] codes
  const uint16_t* s;     // [rows][K/64] bf16 scales
  const uint16_t* b;     // [rows][K/64] bf16 biases
  uint16_t* y;           // [T][ystride] output (row n at column n)
  const uint16_t* res;   // optional residual, same layout as y (may alias it)
  int rows, ystride;
};
struct QGemmArgs {
  QGemmSeg seg[kGemmSegs];
  int nseg;
  const uint16_t* x;     // [T][K] bf16 activations
  int K, T, Np;          // Np: min(T, 256) rounded up to a multiple of 16 (the MMA N)
  int kblocks;           // 64-wide K blocks per split
  int tiles, splits;     // 128-row tiles over all segments, K splits
  int ttiles;            // token tiles of up to 256 (Np tokens each, the last one partial)
  int rows_total;        // sum of the segments' rows (partials row index)
  int stages;            // shared-memory ring depth
  float* part;           // split partials [splits][T][rows_total] f32 (splits > 1)
  uint32_t* counters;    // [tiles], zero between launches
  uint32_t* err;         // bounded-wait failure flag (optional)
  // TMA descriptors (filled by launch_qgemm): each segment's codes as a
  // [rows][K/8] u32 tensor, boxes of 128 rows x 8 words; x as a [T][K] bf16
  // tensor, boxes of Np tokens x 64, landing in the 128-byte swizzle
  alignas(64) CUtensorMap cmap[kGemmSegs];
  alignas(64) CUtensorMap xmap;
};

// Per-token steps of the tensor-core batched-session route (q35_tokens.cu).
struct TokArgs {
  int n;                       // tokens = sessions
  const uint16_t* h_in;        // rms: [n][1024]
  uint16_t* h_out;             // embedding: [n][1024]
  const uint16_t* gain;        // rms gain [1024]
  uint16_t* xn;                // rms output [n][1024]
  const uint32_t* ew;          // embedding codes (non-null: embed the sessions' tokens first)
  const uint16_t* es;
  const uint16_t* eb;
  Ctl* const* ctls;            // [n] sessions' control blocks
  uint32_t* const* seqs;       // [n] sessions' token rings
  float* rope;                 // [n][64] RoPE rows of the step positions
  const uint16_t* raw;         // conv: [n][raw_stride] qkv projections
  int raw_stride;
  uint16_t* conv;              // [n][6144]
  uint16_t* const* hists;      // [n] sessions' conv histories (+ hist_off)
  size_t hist_off;
  const uint16_t* convw;       // [6144][4]
  const uint16_t* y;           // normgate: [n][2048] recurrence output
  const float* zs;             // [n][2048] z * sigmoid(z)
  const uint16_t* gw;          // [128] norm weight
  uint16_t* gated;             // [n][2048]
  const uint16_t* g;           // swiglu: [n][3584] gate
  const uint16_t* u;           // [n][3584] up
  uint16_t* act;               // [n][3584]
  // prompt chunks (one session, n tokens): token t at position p0 + t of seq
  const uint32_t* seq;
  uint32_t p0;
  Ctl* ctl;
};

// Sequence-split exchange buffers of one rank: records [slot][source][cta]
// of kXRec floats (32 dims of o, then m and l) and flags [slot][source][cta].
// Slot = attention layer * 2 + position parity.
constexpr int kMaxSplit = 8;
constexpr int kXSlots = 12;
constexpr int kXCtas = 64;  // combine CTAs: 8 query heads x 8 stripes of 32 dims
constexpr int kXRec = 40;
__host__ __device__ inline size_t x_rec_off(int slot, int src, int cta, int world) {
  return ((size_t(slot) * world + src) * kXCtas + cta) * kXRec;
}
__host__ __device__ inline size_t x_flag_off(int slot, int src, int cta, int world) {
  return (size_t(slot) * world + src) * kXCtas + cta;
}
inline size_t x_recv_bytes(int world) { return size_t(kXSlots) * world * kXCtas * kXRec * 4; }
inline size_t x_flag_bytes(int world) { return size_t(kXSlots) * world * kXCtas * 8; }

struct HeadArgs {
  const uint32_t* w;      // [248320][128]
  const uint16_t* s;
  const uint16_t* b;
  const uint16_t* x;      // hidden before the final norm (or already normed if gain == null)
  const uint16_t* gain;   // final norm gain, or null
  uint16_t* logits;       // [248320]
  float* part;            // [kHeadCtas][2] (max, sum)
  uint32_t* seq;          // token ring (writes seq[pos_step + 1])
  uint32_t* out_tokens;   // writes out_tokens[out_count++]
  uint32_t seq_len;       // entries in seq
  uint32_t out_len;       // entries in out_tokens
  uint16_t* lse_out;      // optional [1]
  Ctl* ctl;
};

// Batched sessions: per-session outputs of the vocabulary head.
constexpr int kMaxSessions = 8;         // exact batched route (CUDA cores)
constexpr int kMaxTensorSessions = 64;  // tensor-core batched route
struct HeadOut {
  uint16_t* logits;     // [248320]
  float* part;          // [kHeadCtas][2]
  uint32_t* seq;        // the session's token ring
  uint32_t* out_tokens; // the session's output ring
  uint32_t seq_len, out_len;
  uint16_t* lse;        // [1]
  Ctl* ctl;             // the session's control block
};
struct HeadBatchArgs {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  const uint16_t* x;      // [n][1024] hidden states before the final norm
  const uint16_t* gain;
  int n;                  // sessions, <= kMaxSessions
  HeadOut out[kMaxSessions];
};

// Prompt chunks on the tensor cores (q35_prompt.cu): T consecutive prompt
// tokens of one session at positions p0 .. p0 + T - 1, with the projections as
// tcgen05 GEMMs over the chunk, the conv and GDN preparation per token, the
// recurrence walking the chunk, and causal flash attention on the tensor cores
// over 128-row blocks (4 query heads x 32 tokens) against 64-key tiles.
constexpr int kPromptChunk = 2048;        // default and largest tokens per chunk
constexpr int kPromptRecSub = 32;         // recurrence staging block (tokens)
constexpr uint32_t kErrPromptWait = 9;    // a bounded wait of the prompt kernels expired
struct PromptArgs {
  int T;                  // tokens in this chunk
  uint32_t p0;            // position of its first token
  int tmax;               // rows of the per-token buffers (a multiple of 32)
  Ctl* ctl;
  // GDN layer
  const uint16_t* raw;    // [T][6144] q | k | v projections
  uint16_t* hist;         // the layer's conv history [3][6144]
  const uint16_t* convw;  // [6144][4]
  uint16_t* conv;         // [T][6144] conv outputs
  const uint16_t* ab;     // [T][32] a (0..15) | b (16..31) projections
  const uint16_t* z;      // [T][2048]
  float* zs;              // [T][2048] z * sigmoid(z)
  const float* a_log;     // [16]
  const uint16_t* dt_bias;// [16]
  float* kq;              // [16][tmax][256] normalised k (0..127) | q (128..255)
  float* gb;              // [16][tmax][2] decay gate, beta
  float* vv;              // [16][8][tmax][16] values by head and 16-row block
  float* state;           // the layer's state [16][128][128]
  uint16_t* y;            // [T][2048] recurrence outputs
  // attention layer
  const uint16_t* q_raw;  // [T][4096] query | gate per head
  const uint16_t* k_raw;  // [T][512]
  const uint16_t* v_raw;  // [T][512]
  const uint16_t* q_gain;
  const uint16_t* k_gain;
  const float* rope;      // [T][64] RoPE rows of the chunk's positions
  uint16_t* qn;           // [8][tmax][256] normalised, rotated queries
  uint16_t* kcache;       // the layer's caches, chain layout of `capacity` positions
  uint16_t* vcache;
  uint32_t capacity;
  int nqb, nsplit;        // 32-token query blocks; key splits per block
  float* opart;           // [2][nqb][nsplit][128][256] unnormalised outputs
  float* oml;             // [2][nqb][nsplit][128][2] (max score, sum of weights)
  float* omax;            // [2][nqb][nsplit][128] each split's row maxima (first pass)
  uint16_t* gated;        // [T][2048]
  // TMA descriptors: queries as [8 heads][T][256] (boxes 4 heads x 32 tokens
  // x 64 dims), keys and values as [128 = 2 heads x 64 chains][capacity / 64
  // slots][256] (boxes 64 chains x 1 slot x 64 dims = 64 consecutive positions)
  alignas(64) CUtensorMap qmap;
  alignas(64) CUtensorMap kmap;
  alignas(64) CUtensorMap vmap;
};

}  // namespace q35
