/*
 * q35 oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A scalar-f32 CPU restatement of the reference engine's batch-1 decode
 * arithmetic (Metal kernels under source/src/kernels/ and the layer wiring in
 * source/src/model.rs), including every BF16 rounding point the reference
 * keeps. It is the checker for the CUDA path: only tests/, the smoke check and
 * the CPU-baseline leg of bench.py may load it. The product (libq35cuda.so and
 * the engine executable) never links or calls it.
 *
 * Parity pin: the reference ships no golden vectors (its MLX fixtures are
 * generated at run time into ignored directories) and its Metal/Rust code
 * cannot run here, so the oracle is pinned against known-answer cases derived
 * from the reference's own audits (tie/plant sets of examples/greedy_audit.rs,
 * edge values of examples/gdn_vector_005.rs) and against closed-form checks;
 * see tests/golden/make_golden.py. Reduction order inside a SIMD group is
 * unspecified on the reference hardware; the oracle uses an xor-butterfly
 * (16,8,4,2,1), which is one admissible order.
 *
 * Conventions: bf16 values travel as uint16_t bit patterns; rounding from
 * f32 is round-to-nearest-even. Transcendentals are evaluated in double and
 * rounded once to f32. Products and sums are separately rounded (no FMA
 * contraction) except where the reference writes fma() explicitly.
 */
#ifndef Q35_ORACLE_H
#define Q35_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

void orc_set_threads(int n);
int orc_get_threads(void);

/* ---- elementwise / small ops ---- */
uint16_t orc_f2bf(float f);
float orc_bf2f(uint16_t h);
float orc_sigmoid_bf(float x);
float orc_softplus_bf(float x);
/* the f32 exp taken for the reference's fast::exp */
float orc_fexp(float x);

/* embedding_q4, linear.metal:11-24 */
void orc_embedding_q4(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                      uint32_t token, int K, uint16_t* out);
/* qmv_q4 / qmv_add_q4, linear.metal:28-123. residual may be NULL. */
/* the tensor-core routes' matvec: weights bf16(s q + b), exact dot products (f32 out) */
void orc_qmv_gemm_f32(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x, int N, int K,
                      float* y);
void orc_qmv_q4(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                const uint16_t* x, const uint16_t* residual, int N, int K, uint16_t* y);
/* f32 value before the bf16 store (for tolerance tests) */
void orc_qmv_q4_f32(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                    const uint16_t* x, int N, int K, float* y);
/* rms_norm_bf16, linear.metal:300-331 (256 threads x 4 values) */
void orc_rms_norm(const uint16_t* x, const uint16_t* gain, int cols, float eps, uint16_t* out);
/* swiglu_bf16, linear.metal:382-396 */
void orc_swiglu(const uint16_t* gate, const uint16_t* up, int n, uint16_t* out);

/* gdn_input_g16 tail (conv, history shift, q/k norm, gates), gdn_input.metal:412-460 */
void orc_gdn_conv_prepare(const uint16_t* raw_qkv, const uint16_t* a_raw, const uint16_t* b_raw,
                          uint16_t* history, const uint16_t* conv_w, const float* a_log,
                          const uint16_t* dt_bias, uint16_t* conv_out, float* g, uint16_t* beta);
/* gdn_recur, gdn.metal:176-228 (T=1) */
void orc_gdn_recur(const uint16_t* conv_qkv, const float* g, const uint16_t* beta,
                   float* state, uint16_t* y);
/* gdn_norm_gate, gdn.metal:230-255 */
void orc_gdn_norm_gate(const uint16_t* y, const uint16_t* z, const uint16_t* w, uint16_t* out);
/* whole single-token GDN mixer after the input projections (config 2):
 * conv/prepare -> recurrence -> gated norm -> out_proj + residual.
 * residual may be NULL (then out = bf16(out_proj)). */
void orc_gdn_step(const uint16_t* raw_qkv, const uint16_t* z, const uint16_t* a_raw,
                  const uint16_t* b_raw, uint16_t* history, const uint16_t* conv_w,
                  const float* a_log, const uint16_t* dt_bias, float* state,
                  const uint16_t* norm_w, const uint32_t* ow, const uint16_t* os,
                  const uint16_t* ob, const uint16_t* residual, uint16_t* out);

/* attn_prepare_qkv_decode, attention.metal:262-313. Writes query[2048] and
 * appends K/V at position pos of caches laid out [2][capacity][256]. */
void orc_attn_prepare(const uint16_t* q_raw, const uint16_t* k_raw, const uint16_t* v_raw,
                      const uint16_t* q_gain, const uint16_t* k_gain, uint32_t pos,
                      uint32_t capacity, uint16_t* query, uint16_t* kcache, uint16_t* vcache);
/* decode attention + output gate: sdpa_vector (len<1024, attention_decode.metal:51-213
 * then attn_gate attention.metal:133-151) or the 64-block split route
 * (attention_decode.metal:215-431 + :830-891). Writes gated[2048]. */
void orc_attn_decode_gate(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache,
                          uint32_t len, uint32_t capacity, const uint16_t* q_raw, uint16_t* gated);
/* The same output under the engine's sequence split over `world` ranks
 * (positions p % world == r on rank r, f32 chain partials, per-rank records
 * merged in rank order; world 1 = orc_attn_decode_gate). */
void orc_attn_decode_gate_split(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache,
                                uint32_t len, uint32_t capacity, int world, const uint16_t* q_raw,
                                uint16_t* gated);
/* f32 attention output before rounding (for tolerance tests), o[8*256] */
/* the tensor-core prompt route's attention (f32, before the gate) */
void orc_attn_flash_f32(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache,
                        uint32_t len, uint32_t capacity, float* o);
/* the prompt route's attention followed by the output gate */
void orc_attn_flash_gate(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache, uint32_t len,
                         uint32_t capacity, const uint16_t* q_raw, uint16_t* gated);
void orc_attn_decode_f32(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache,
                         uint32_t len, uint32_t capacity, float* o);

/* head_lse_g8 + head_lse_tail, head_lse.metal:11-98. Returns the token;
 * writes bf16 logits[N] and the bf16 lse bit pattern. */
uint32_t orc_head(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x,
                  int N, int K, uint16_t* logits, uint16_t* lse_out);
/* greedy tail alone on given logits (lse computed the reference way) */
uint32_t orc_greedy(const uint16_t* logits, int N, uint16_t* lse_out);
/* greedy with a given lse: lowest id among maxima of bf16(l - lse) */
uint32_t orc_greedy_with_lse(const uint16_t* logits, int N, uint16_t lse);

/* logits of the reference's greedy audit, case si (examples/greedy_audit.rs) */
void orc_xorshift_logits(uint64_t* seed, int si, int N, uint16_t* out);

/* ---- full model (model.rs rows=1 route) ---- */
typedef struct orc_model orc_model;
typedef struct orc_session orc_session;
orc_model* orc_model_load(const char* dir, char* err, int err_len);
void orc_model_free(orc_model* m);
orc_session* orc_session_new(orc_model* m, uint32_t capacity);
void orc_session_free(orc_session* s);
void orc_session_reset(orc_session* s);
uint32_t orc_session_position(const orc_session* s);
/* consume `token` at the current position; if want_head, returns the greedy
 * next token (and keeps logits), else returns 0xffffffff. */
/* projections and head of later steps with the engine's tensor-core route's
 * numerics (weights dequantised to bf16, dot products exact then rounded) */
void orc_session_set_gemm(orc_session* s, int on);
/* Tokens per GEMM launch of the engine route being restated (batch members,
 * prompt-chunk tokens): with the launch's row tiles it fixes the K split. */
void orc_session_set_gemm_tokens(orc_session* s, int tokens);
/* The prompt chunk (first position, token count) the next steps belong to:
 * sets the GEMM token count, and in flash mode the attention restates the
 * prompt route exactly (orc_attn_flash_tc_gate). */
void orc_session_set_chunk(orc_session* s, uint32_t p0, uint32_t tokens);
/* The prompt route's gated attention, exactly (the kernel's splits, fexp
 * weights, MMA accumulation), for the token at `pos` of the chunk (p0c, T). */
void orc_attn_flash_tc_gate(const uint16_t* query, const uint16_t* kcache, const uint16_t* vcache, uint32_t pos,
                            uint32_t capacity, uint32_t p0c, uint32_t T, const uint16_t* q_raw, uint16_t* gated);
/* The engine's tensor-core GEMM on T tokens (x [T][K]): y [T][N] before the
 * bf16 rounding, for a launch of `tiles` 128-row tiles (0: this matrix alone). */
void orc_qgemm_tc(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x, int T, int N,
                  int K, int tiles, float* y);
/* One 16-wide K step of the tensor core's bf16 MMA (f32 accumulator):
 * acc + sum a[i] b[i] with the measured alignment and truncation. */
float tc_step(float acc, const float* a, const float* b);
/* attention of later steps as the tensor-core prompt route's (attn_f32_flash) */
void orc_session_set_flash(orc_session* s, int on);
/* attention of later steps as the engine's sequence split over `world` ranks */
void orc_session_set_split(orc_session* s, int world);
uint32_t orc_session_step(orc_session* s, uint32_t token, int want_head);
void orc_session_logits(const orc_session* s, uint16_t* out); /* [248320] */
uint16_t orc_session_lse(const orc_session* s);
/* hidden state after the final norm, bf16[1024] */
void orc_session_final_hidden(const orc_session* s, uint16_t* out);
/* teacher-forcing import of a device state dump: per attention layer a
 * (li=0..5) K and V caches [2][cap_src][256] of which `pos` positions are
 * copied; per GDN layer (gi=0..17) state f32[16*128*128] and history
 * bf16[3*6144]. */
void orc_session_export(const orc_session* s, uint16_t* kv, float* state, uint16_t* hist);
void orc_session_import(orc_session* s, uint32_t pos, uint32_t cap_src,
                        const uint16_t* const* kcaches, const uint16_t* const* vcaches,
                        const float* const* states, const uint16_t* const* histories);

#ifdef __cplusplus
}
#endif
#endif
