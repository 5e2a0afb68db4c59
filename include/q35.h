/*
 * q35 — C ABI of the B200 decode engine for the Qwen3.5-0.8B-class 4-bit
 * hybrid model (libq35cuda.so).
 *
 * This is the boundary the reference's Rust host would bind through FFI.
 * Paths below are relative to the reference's source/ tree.
 *
 *   session API  <->  Model::load / Model::generate / Model::cancelled
 *                     (src/model.rs:28-34, :37-92, :97-122, :123-180)
 *   op API       <->  the Metal entry points the model dispatches through
 *                     Gpu::dispatch (src/gpu.rs:69-79)
 *
 * Conventions: bf16 tensors are uint16_t bit patterns; device pointers are
 * CUDA device addresses; `stream` is a cudaStream_t passed as void* (NULL =
 * legacy default stream). Every function returns 0 on success or a negative
 * Q35_E* code. Op-level calls allocate nothing: they borrow the caller's
 * buffers (including any workspace) and enqueue work on `stream`.
 */
#ifndef Q35_H
#define Q35_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q35_OK 0
#define Q35_EINVAL (-1)    /* validation failed; session state untouched */
#define Q35_ECUDA (-2)     /* device error; session state was reset */
#define Q35_ECANCEL (-3)   /* q35_cancel() observed ("input disconnected") */
#define Q35_EIO (-4)       /* model directory / file / format error */
#define Q35_ENOMEM (-5)
#define Q35_ETIMEOUT (-6)  /* a bounded device wait expired; state was reset */
#define Q35_ENCCL (-7)

#define Q35_VOCAB 248320u
#define Q35_HIDDEN 1024u
#define Q35_DEFAULT_CAPACITY 262144u /* model.rs:8 */

typedef struct q35_session q35_session;

typedef struct q35_opts {
  uint32_t capacity;     /* context capacity in tokens (0 -> 262144); multiple of 64 */
  uint32_t decode_batch; /* decode steps per CUDA-graph launch (0 -> 8) */
  uint32_t prefill_batch;/* prompt steps per CUDA-graph launch (0 -> 16) */
  uint32_t flags;        /* Q35_FLAG_* bits, 0 by default */
  uint32_t prompt_chunk; /* tokens per tensor-core prompt chunk (0 -> 2048); a
                            multiple of 32 in 32..2048 */
} q35_opts;

/* Consume prompts one token per step (the decode step without the head)
 * instead of in chunks of 16 tokens. Both give bit-identical state; the
 * chunked route reads each weight once per chunk. */
#define Q35_FLAG_TOKEN_BY_TOKEN_PROMPT 1u

/* Consume prompts on the tensor cores, as the reference's prefill does
 * (model.rs:100-110, :189-198): chunks of prompt_chunk tokens with every
 * projection a tcgen05 GEMM over the chunk and causal flash attention on the
 * tensor cores (bf16 attention weights). The state after the prompt then
 * differs from the decode route's within the GEMM/flash-attention tolerance
 * rather than bit for bit; decoding is unchanged. Ignored under a sequence
 * split (those prompts take the decode route). */
#define Q35_FLAG_TENSOR_PROMPT 2u

/* ---------------------------------------------------------------------- */
/* Session API                                                             */
/* ---------------------------------------------------------------------- */

/* Load MODEL_DIR (config.json + *.safetensors in the MLX layout, 694
 * language_model.model.* tensors) onto `device`, allocate every buffer and
 * capture the decode graphs. Replaces Model::load (model.rs:37-92) and
 * Weights::load (weights.rs:11-44). On failure *out is NULL and, if err is
 * non-NULL, a message is copied into err[0..err_len). */
int q35_open(const char* model_dir, int device, const q35_opts* opts, q35_session** out,
             char* err, size_t err_len);

/* Model::generate (model.rs:97-122). reset != 0: discard state, consume
 * prompt[0..n_prompt) (n_prompt >= 1) and emit max_tokens greedy ids.
 * reset == 0: n_prompt must be 0; first consume the last emitted token, then
 * emit max_tokens ids. out_tokens has room for max_tokens ids. Validation
 * errors (empty prompt, capacity, id >= vocab, no continuation state) return
 * Q35_EINVAL and leave the state intact; device errors and cancellation
 * reset the session (model.rs:166-178). */
int q35_generate(q35_session* s, const uint32_t* prompt, size_t n_prompt, size_t max_tokens,
                 int reset, uint32_t* out_tokens);

/* Model::cancelled (main.rs:23-24, model.rs:133-144): thread-safe; the
 * running q35_generate drains its queued work and returns Q35_ECANCEL. */
void q35_cancel(q35_session* s);

/* Message of the last failure on this session (never NULL). */
const char* q35_last_error(const q35_session* s);

void q35_close(q35_session* s);

/* Tokens consumed so far (Model::position, model.rs:32). */
uint32_t q35_position(const q35_session* s);

/* Context capacity of the session in tokens (model.rs:8, CAPACITY): the
 * bound of generate's "invalid output length" and "context capacity
 * exceeded" checks (model.rs:98-113). */
uint32_t q35_capacity(const q35_session* s);

/* The pending token (Model::pending, model.rs:32): the last emitted id, which
 * the next q35_generate(reset=0) consumes first. Q35_EINVAL when the session
 * holds no continuation state. */
int q35_pending(const q35_session* s, uint32_t* token);

/* Validates session options as q35_open does, without a device or a model
 * (host arithmetic only): Q35_OK, or Q35_EINVAL with the message q35_open
 * would give (e.g. "capacity must be a positive multiple of 64"). No
 * counterpart in the reference, whose capacity is a constant. */
int q35_check_opts(const q35_opts* opts, char* err, size_t err_len);

/* Kernel launches the session's decode steps have enqueued since the last
 * reset (the kernel nodes of each replayed decode graph, counted when the
 * graph was captured); reset != 0 clears the count after reading it.
 * Benchmark aid, no counterpart in the reference. */
int q35_launch_count(q35_session* s, int reset, uint64_t* launches);

/* Copy the device state to host memory for checking: per attention layer
 * (6) K and V caches, converted to position order and truncated to the first
 * `pos` positions (layout [2][pos][256] each), per GDN layer (18) recurrent state
 * f32 [16][128][128] and conv history bf16 [3][6144]. Buffers must hold
 * 6*2*2*pos*256*2 bytes (kv), 18*16*128*128*4 (state), 18*3*6144*2 (hist). */
int q35_dump_state(q35_session* s, uint16_t* kv, float* state, uint16_t* hist);

/* bf16 logits [248320] and lse of the last emitted token. */
int q35_last_logits(q35_session* s, uint16_t* logits, uint16_t* lse);

/* Decode-only timing helpers for benchmarks: run `steps` greedy decode steps
 * on the current state (as q35_generate with reset=0 would) but leave the
 * tokens on the device; returns the device time in milliseconds. */
int q35_decode_timed(q35_session* s, size_t steps, float* ms);

/* Session copy (no counterpart in the reference): dst takes src's whole
 * decode state (position, continuation token, token history, KV cache,
 * recurrent state, conv history, last logits), so both continue identically;
 * e.g. one prompt consumed once and decoded by several sessions. Same device,
 * model directory and capacity; device-to-device copies on dst's stream. */
int q35_session_copy(q35_session* dst, q35_session* src);

/* Teacher forcing (test and evaluation aid, no reference counterpart):
 * replace the pending token, i.e. the last emitted id that the next
 * q35_generate(reset=0) consumes first. Needs a continuation state. */
int q35_force_pending(q35_session* s, uint32_t token);

/* Sequence-split attention (the reference runs one GPU):
 * one decode stream over `world` GPUs, one session and one process per GPU,
 * all opened on the same model with the same capacity. Every rank runs the
 * replicated non-attention layers; rank r keeps the K/V of positions p with
 * p % world == r, and each attention combine exchanges the ranks' partial
 * (max, sum, unnormalised o) over NVLink: every rank writes its record into
 * every rank's receive buffer (CUDA IPC mappings) and merges all records in
 * rank order, so all ranks emit the same tokens. Attention always takes the
 * 64-chain route here, so tokens agree with a single-GPU session within the
 * floating-point tolerance rather than bit for bit.
 * Set-up: q35_split_prepare on every rank (allocates the exchange buffer and
 * returns its IPC handle), exchange the handles between the processes (any
 * channel), then q35_split_connect with all `world` handles in rank order
 * (maps the peers' buffers, recaptures the graphs, resets the state). After
 * that every rank must make the same q35_generate calls in the same order;
 * a rank whose peers stop answering gets Q35_ETIMEOUT after about 10 s.
 * q35_split_world returns the connected world size (1 when not split). */
#define Q35_SPLIT_HANDLE_BYTES 64
int q35_split_prepare(q35_session* s, int rank, int world, void* handle);
int q35_split_connect(q35_session* s, const void* handles);
int q35_split_world(const q35_session* s);
/* Bound, in milliseconds (1..600000), of each attention combine's wait for
 * the peers' records; 10 s unless set. Call before q35_split_connect (the
 * decode graphs are captured there). A wait that runs out makes the request
 * fail with Q35_ETIMEOUT and resets the session; the peers' next exchanges
 * (which wait for this rank) run out the same way. */
int q35_split_set_wait(q35_session* s, uint32_t ms);

/* Batched sessions (no counterpart in the reference, whose engine serves one
 * stream): 1..8 sessions of one device, each already holding a continuation
 * state (a q35_generate call returned Q35_OK on it), decoded together. Each
 * batched step streams the weights once for all sessions; every session
 * keeps its own KV cache, recurrent state, position and token ring, and emits
 * exactly the tokens and logits it would emit decoding alone. The batch keeps
 * pointers to the sessions: destroy the batch before any of them, and do not
 * call q35_generate on a member while a batch call runs. q35_generate with
 * reset=0 continues a member after a batch call, as after its own. */
typedef struct q35_batch q35_batch;
int q35_batch_create(q35_session** sessions, int n, q35_batch** out, char* err, size_t err_len);
/* Q35_BATCH_TENSOR_CORES: 1..64 sessions, every projection and the head as a
 * Q4 GEMM on the tensor cores (q35_op_qgemm_q4's arithmetic: weights
 * dequantised to bf16, float32 accumulation in the tensor core's order), the
 * other steps as in decode; the sessions' attention and recurrences run in
 * one launch each. Results agree with the exact route within floating-point
 * tolerance, not bit for bit. Without the flag: the exact route, 1..8
 * sessions. */
#define Q35_BATCH_TENSOR_CORES 1u
int q35_batch_create_ex(q35_session** sessions, int n, uint32_t flags, q35_batch** out, char* err,
                        size_t err_len);
/* `steps` greedy steps for every member; out_tokens is [n][steps] (row t =
 * session t). Fails (Q35_EINVAL, nothing run) when a member lacks a
 * continuation state or would pass its capacity. */
int q35_batch_decode(q35_batch* b, size_t steps, uint32_t* out_tokens);
/* As q35_batch_decode, tokens left on the device; device time in ms. */
int q35_batch_decode_timed(q35_batch* b, size_t steps, float* ms);
const char* q35_batch_last_error(const q35_batch* b);
/* Kernel launches of the batch's decode graphs since the last reset (as
 * q35_launch_count). */
int q35_batch_launch_count(q35_batch* b, int reset, uint64_t* launches);
void q35_batch_destroy(q35_batch* b);

/* Device-clock timing of the attention launches (benchmark aid, no
 * counterpart in the reference): reads the summed launch time in
 * microseconds and the launch count since the last reset; reset > 0 clears
 * and enables the timer, reset == 0 clears and disables it, reset < 0 only
 * reads. A launch lasts from its earliest post-dependency start to the end of
 * its last CTA. */
int q35_attn_timing(q35_session* s, int reset, double* total_us, uint32_t* launches);

/* Device-clock timing of the matvec launches, on the same switch as
 * q35_attn_timing (whose reset clears both): the summed launch time in
 * microseconds, the launch count and the launches' summed algorithmic bytes
 * (rows x (K/2 code bytes + K/16 scale and bias bytes)) since the last reset.
 * Benchmark aid, no counterpart in the reference. */
int q35_qmv_timing(q35_session* s, double* total_us, uint32_t* launches, double* weight_bytes);

/* ---------------------------------------------------------------------- */
/* Op API (device pointers, caller-owned, nothing allocated)               */
/* ---------------------------------------------------------------------- */

/* qmv_q4 / qmv_add_q4 (kernels/linear.metal:28-123): y[N] = bf16(W x), or
 * bf16(residual + bf16(W x)) when residual is non-NULL (residual may alias y).
 * W: codes [N][K/8] u32, scales/biases [N][K/64] bf16; K in {1024, 2048, 3584}
 * (any multiple of 512 up to 4096); x [K] bf16. */
int q35_op_qmv_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                  const uint16_t* x, const uint16_t* residual, uint16_t* y, int n, int k,
                  void* stream);

/* Batched Q4 matmul on the tensor cores (tcgen05; the batched-session route,
 * in the place of the reference's quantised matmul qmm_q4_nax,
 * kernels/linear_nax.metal:1096-1139): y[t][n] = bf16(sum_k W[n][k] x[t][k]),
 * or bf16(residual[t][n] + bf16(.)) when residual is non-NULL (may alias y),
 * for t < tokens (1..4096), with W dequantised as bf16(s*q + b). x [tokens][k]
 * bf16, y [tokens][n]; n up to 524,288; k a multiple of 512 up to 4096; w, x, scales, biases and
 * workspace 16-byte aligned. The float32 accumulation runs in
 * the tensor core's order, so results match a float32 reference within
 * tolerance rather than the matvec bit for bit. workspace: at least
 * q35_op_qgemm_workspace_bytes(tokens, n, k) bytes (0 = invalid shape). */
/* Prompt chunks on the tensor cores, one layer's steps over `tokens` (1..2048)
 * consecutive prompt tokens, for tests and other hosts. Workspace: at least
 * q35_op_prompt_workspace_bytes(tokens, capacity) bytes (capacity 0 for the
 * GDN op; 0 = invalid shape), 16-byte aligned.
 *
 * q35_op_prompt_gdn: the GDN conv, preparation, recurrence and gated norm of
 * the prefill (gdn.metal gdn_conv :33-52, gdn_history :56-71, gdn_prepare
 * :75-114, the multi-row gdn_recur loop :176-228, gdn_norm_gate :230-255):
 * raw_qkv [T][6144], z [T][2048], ab [T][32] (a | b projections), history
 * [3][6144] and state [16][128][128] f32 updated in place, conv_w [6144][4],
 * a_log [16] f32, dt_bias [16], norm_w [128]; gated [T][2048]. Each token's
 * arithmetic is the decode step's, so results equal T decode steps bit for bit.
 *
 * q35_op_prompt_attention: per-head q/k norm, partial RoPE and the K/V append
 * of positions p0 .. p0 + T - 1 (attention.metal:72-131), causal flash
 * attention on the tensor cores (attention_prefill.metal:1830-2258) and the
 * output gate (attention.metal:140-150): q_raw [T][4096] (query | gate per
 * head), k_raw and v_raw [T][512], caches in the chain layout of `capacity`
 * positions (as q35_op_attn_decode), gated [T][2048]. Attention weights are
 * bf16 and sums run in the tensor core's order (tolerance, not bit-exact). */
size_t q35_op_prompt_workspace_bytes(uint32_t tokens, uint32_t capacity);
int q35_op_prompt_gdn(const uint16_t* raw_qkv, const uint16_t* z, const uint16_t* ab, uint16_t* history,
                      const uint16_t* conv_w, const float* a_log, const uint16_t* dt_bias, float* state,
                      const uint16_t* norm_w, uint32_t tokens, uint16_t* gated, void* workspace,
                      size_t workspace_bytes, void* stream);
int q35_op_prompt_attention(const uint16_t* q_raw, const uint16_t* k_raw, const uint16_t* v_raw,
                            const uint16_t* q_gain, const uint16_t* k_gain, uint16_t* kcache, uint16_t* vcache,
                            uint32_t capacity, uint32_t p0, uint32_t tokens, uint16_t* gated, void* workspace,
                            size_t workspace_bytes, void* stream);

size_t q35_op_qgemm_workspace_bytes(uint32_t tokens, uint32_t n, uint32_t k);
int q35_op_qgemm_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                    uint32_t tokens, uint32_t n, uint32_t k, const uint16_t* residual, uint16_t* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/* embedding_q4 (kernels/linear.metal:11-24): out[K] = bf16(s*q + b) of row `token`. */
int q35_op_embedding_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        uint32_t token, int k, uint16_t* out, void* stream);

/* rms_norm_bf16 (kernels/linear.metal:300-331) for one 1024-wide row, eps 1e-6. */
int q35_op_rms_norm(const uint16_t* x, const uint16_t* gain, uint16_t* out, void* stream);

/* Single-token gated-delta-net mixer after the input projections:
 * gdn_input_g16's conv/prepare tail (kernels/gdn_input.metal:412-460),
 * gdn_recur (kernels/gdn.metal:176-228), gdn_norm_gate (:230-255) and the
 * out_proj qmv_add_q4 (model.rs:265). raw_qkv [6144], z [2048], a/b [16] bf16;
 * history [3][6144] bf16 and state [16][128][128] f32 are updated in place;
 * conv_w [6144][4] bf16, a_log [16] f32, dt_bias [16] bf16, norm_w [128] bf16;
 * out_proj Q4 [1024][2048]; residual may be NULL. Workspace: at least
 * q35_op_gdn_workspace_bytes() bytes of device memory. */
size_t q35_op_gdn_workspace_bytes(void);
int q35_op_gdn_step(const uint16_t* raw_qkv, const uint16_t* z, const uint16_t* a_raw,
                    const uint16_t* b_raw, uint16_t* history, const uint16_t* conv_w,
                    const float* a_log, const uint16_t* dt_bias, float* state,
                    const uint16_t* norm_w, const uint32_t* ow, const uint16_t* os,
                    const uint16_t* ob, const uint16_t* residual, uint16_t* out,
                    void* workspace, void* stream);

/* Gated GQA decode attention for one token at position `pos`:
 * attn_prepare_qkv_decode (kernels/attention.metal:262-313) appends the
 * token's K/V at `pos`, then split-K attention over keys 0..pos
 * (kernels/attention_decode.metal:215-431) and the combine with the BF16
 * output gate (:830-891). q_raw [8][512] (query | gate), k_raw/v_raw
 * [2][256], q/k norm gains [256]; gated [8][256] bf16. The caches are
 * chain-major bf16 [2 kv heads][64][capacity/64][256]: position p of a kv
 * head lives at chain p % 64, slot p / 64 (capacity a multiple of 64,
 * pos < capacity), so each of the reference's 64 key blocks (keys b, b+64,
 * ...) is contiguous. q_raw, k_raw, v_raw, the gains and both caches must be
 * 16-byte aligned (Q35_EINVAL otherwise). */
size_t q35_op_attn_workspace_bytes(void);
int q35_op_attn_decode(const uint16_t* q_raw, const uint16_t* k_raw, const uint16_t* v_raw,
                       const uint16_t* q_gain, const uint16_t* k_gain, uint16_t* kcache,
                       uint16_t* vcache, uint32_t capacity, uint32_t pos, uint16_t* gated,
                       void* workspace, void* stream);

/* Status of an op call's bounded device waits. Every op runs
 * asynchronously; a wait inside it that gives up (after 2^24 polls) lets the
 * kernel finish and records a site code in the op's workspace instead of
 * hanging the stream. This waits for `stream`, then reads that word:
 * Q35_OK, or Q35_ETIMEOUT with *site (may be NULL) set to the code; the word
 * is cleared by the op's next call on the same workspace. kind:
 * Q35_OPWS_CTL for the workspaces of q35_op_gdn_step, q35_op_attn_decode,
 * q35_op_head_argmax, q35_op_greedy, q35_op_prompt_gdn and
 * q35_op_prompt_attention (a control block first), with workspace NULL for
 * q35_op_attn_decode_noalloc's scratch on the current device (after its
 * first call there); Q35_OPWS_QGEMM for q35_op_qgemm_q4's workspace. No
 * counterpart in the reference, whose Metal waits are unbounded. */
#define Q35_OPWS_CTL 0u
#define Q35_OPWS_QGEMM 1u
int q35_op_status(const void* workspace, uint32_t kind, uint32_t* site, void* stream);

/* Allocation-free form of q35_op_attn_decode, for callers that cannot call
 * cudaMalloc or hand out a workspace (no counterpart in the reference: its
 * Metal host allocates every buffer itself). Same arguments and results as
 * q35_op_attn_decode, minus the workspace: the scratch is a 576 KiB array in
 * the library's device image, held by every device that loads the library
 * until exit (this op uses 528,896 bytes of it at any context length; the
 * build fails if the layout outgrows the array). The first call on a device
 * looks up the array's address and sets kernel attributes, so make it before
 * any stream capture; the address is kept per device number, so calls after
 * a cudaDeviceReset of that device are unsupported.
 * All calls on a device share the array: calls that overlap on the GPU race.
 * Rejected arguments return Q35_EINVAL with a message in err (may be NULL). */
int q35_op_attn_decode_noalloc(const uint16_t* q_raw, const uint16_t* k_raw,
                               const uint16_t* v_raw, const uint16_t* q_gain,
                               const uint16_t* k_gain, uint16_t* kcache, uint16_t* vcache,
                               uint32_t capacity, uint32_t pos, uint16_t* gated, char* err,
                               size_t err_len, void* stream);

/* Final RMSNorm (gain may be NULL to skip it), vocabulary projection of the
 * tied Q4 embedding [248320][1024] and greedy selection
 * (kernels/head_lse.metal:11-98, linear.metal:300-331): logits [248320]
 * bf16, token [1] u32, lse [1] bf16 (may be NULL). */
size_t q35_op_head_workspace_bytes(void);
int q35_op_head_argmax(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                       const uint16_t* x, const uint16_t* gain, uint16_t* logits,
                       uint32_t* token, uint16_t* lse, void* workspace, void* stream);

/* greedy_bf16 (kernels/linear.metal:400-449) on given bf16 logits [248320]:
 * lse = bf16(logsumexp), token = lowest id among the maxima of
 * bf16(logit - lse). Workspace: q35_op_head_workspace_bytes(). */
int q35_op_greedy(const uint16_t* logits, uint32_t* token, uint16_t* lse, void* workspace,
                  void* stream);

/* ---------------------------------------------------------------------- */
/* Utility (no counterpart in the reference)                               */
/* ---------------------------------------------------------------------- */

/* Write a seeded random-init model directory in the MLX layout the loader
 * expects: config.json + model.safetensors with the 694 tensors of the
 * model (all linears Q4 affine group-64 quantised from N(0, 0.02)). */
int q35_write_synthetic_model(const char* dir, uint64_t seed, char* err, size_t err_len);

/* Library build string. */
const char* q35_version(void);

/* ---------------------------------------------------------------------- */
/* Diagnostics for failure-detection tests (no counterpart in the          */
/* reference, whose Metal waits are unbounded)                            */
/* ---------------------------------------------------------------------- */

/* Runs the bounded mbarrier wait that every kernel uses on a barrier nothing
 * completes, giving up after `polls` polls: returns Q35_ETIMEOUT and leaves
 * the wait's site code in *err_dev (a 4-byte device word), with the device
 * context still usable. */
int q35_diag_bounded_wait(uint32_t polls, uint32_t* err_dev, void* stream);

/* Records an expired device wait with site code `site` in the session's
 * control block, as a kernel whose bounded wait ran out would: the next
 * continuation request then fails with Q35_ETIMEOUT and resets the session
 * (model.rs:166-178). Host-side fault injection; runs no faulting code. */
int q35_diag_inject_device_error(q35_session* s, uint32_t site);

#ifdef __cplusplus
}
#endif
#endif /* Q35_H */
