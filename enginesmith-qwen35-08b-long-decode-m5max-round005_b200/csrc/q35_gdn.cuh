// Gated delta net and attention-prologue arithmetic shared by the decode
// step and the prompt paths, so all evaluate exactly the same operations in
// the same order (the oracle's restatement of gdn_input.metal / gdn.metal /
// attention.metal).
#pragma once
#include "q35_qmv.cuh"

namespace q35 {

// gdn_input.metal:419-431: 4-tap causal conv (tap 3 = current token), BF16
// boundary, SiLU with the BF16-stepped sigmoid. Returns the conv output; the
// caller shifts the history (h0 <- h1, h1 <- h2, h2 <- raw).
Q35_DEV uint16_t gdn_conv_value(uint16_t h0, uint16_t h1, uint16_t h2, uint16_t raw, const uint16_t* w4) {
  float acc = 0.0f;
  acc = fmaf(bf2f(h0), bf2f(w4[0]), acc);
  acc = fmaf(bf2f(h1), bf2f(w4[1]), acc);
  acc = fmaf(bf2f(h2), bf2f(w4[2]), acc);
  acc = fmaf(bf2f(raw), bf2f(w4[3]), acc);
  const float xq = bfr(acc);
  return f2bf(__fmul_rn(xq, sigmoid_bf(xq)));
}

// gdn_input.metal:433-441 for one warp: q (is_q) or k of head h from the conv
// outputs `conv` [6144]; lane l owns channels 4l..4l+3 of the head. Writes
// the 128 normalised values (as f32) to dst.
Q35_DEV void gdn_qk_norm(const uint16_t* conv, int h, bool is_q, int lane, float* dst) {
  const int base = is_q ? h * 128 : 2048 + h * 128;
  const float4 v4 = bf4(*reinterpret_cast<const uint2*>(conv + base + 4 * lane));
  const float v[4] = {v4.x, v4.y, v4.z, v4.w};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  ss = warp_sum(ss);
  const float inv = drsqrtf(__fadd_rn(__fmul_rn(ss, 0.0078125f), 1.0e-6f / 128.0f));
  const float scale = is_q ? 0.0078125f : bfr(0.08838834764831845f);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[4 * lane + i] = bfr(__fmul_rn(bfr(__fmul_rn(v[i], inv)), scale));
}

// gdn_input.metal:454-459: decay gate g = exp(-exp(A_log) * softplus_bf(bf16(a + dt_bias)))
// (e1 = exp(A_log) is passed in) and write strength beta = bf16(sigmoid_bf(b)).
Q35_DEV float gdn_gate(uint16_t a_raw, uint16_t dt_bias, float e1) {
  const float ax = bfr(__fadd_rn(bf2f(a_raw), bf2f(dt_bias)));
  return dexpf(__fmul_rn(-e1, softplus_bf(ax)));
}
Q35_DEV float gdn_beta(uint16_t b_raw) { return bfr(sigmoid_bf(bf2f(b_raw))); }

// gdn.metal:246-253: the output gate z * sigmoid(z) with sigmoid in plain f32
// (1 / (1 + e^|z|) mirrored by sign), as the norm-gate prologue forms it.
Q35_DEV float gdn_zgate(float z) {
  const float sy = __fdiv_rn(1.0f, __fadd_rn(1.0f, dexpf(fabsf(z))));
  const float sig = z < 0.0f ? sy : __fsub_rn(1.0f, sy);
  return __fmul_rn(z, sig);
}

// gdn.metal:192-225 for one value row, T = 1: 4 lanes per row (lane quarter
// r owns keys 32r..32r+31, state in s[32]); S *= g; mem = S k (eight
// four-term partials, then shuffle-xor 1, 2); delta = (v - mem) * beta;
// S += k delta; out = S q (same reduction). Returns out on all 4 lanes.
Q35_DEV float gdn_row_step(float (&s)[32], const float* kk, const float* qq, float gt, float beta,
                           float vval) {
  float part[8];
#pragma unroll
  for (int pb = 0; pb < 8; ++pb) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = pb * 4 + i;
      s[e] = __fmul_rn(s[e], gt);
      acc = __fadd_rn(acc, __fmul_rn(s[e], kk[e]));
    }
    part[pb] = acc;
  }
  float memory = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3])),
                           __fadd_rn(__fadd_rn(part[4], part[5]), __fadd_rn(part[6], part[7])));
  memory = __fadd_rn(memory, __shfl_xor_sync(0xffffffffu, memory, 1));
  memory = __fadd_rn(memory, __shfl_xor_sync(0xffffffffu, memory, 2));
  const float delta = __fmul_rn(__fsub_rn(vval, memory), beta);
#pragma unroll
  for (int pb = 0; pb < 8; ++pb) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = pb * 4 + i;
      s[e] = __fadd_rn(s[e], __fmul_rn(kk[e], delta));
      acc = __fadd_rn(acc, __fmul_rn(s[e], qq[e]));
    }
    part[pb] = acc;
  }
  float out = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3])),
                        __fadd_rn(__fadd_rn(part[4], part[5]), __fadd_rn(part[6], part[7])));
  out = __fadd_rn(out, __shfl_xor_sync(0xffffffffu, out, 1));
  out = __fadd_rn(out, __shfl_xor_sync(0xffffffffu, out, 2));
  return out;
}

// gdn_row_step with 8 lanes per value row, in pieces: lane octant r8 owns
// keys 16 r8 .. 16 r8 + 15, i.e. partials 4 (r8 & 1) .. 4 (r8 & 1) + 3 of lane
// quarter r8 / 2. Each lane sums its four partials as that quarter's half of
// the tree ((p0 + p1) + (p2 + p3)), shuffle-xor 1 joins the halves, and xor 2
// and 4 take the quarters' xor 1 and 2: the same additions in the same
// association (a + b = b + a exactly), so memory (gdn_decay_dot8 reduced by
// gdn_reduce8), delta = (v - memory) * beta, and out (gdn_update_dot8
// reduced) equal gdn_row_step's results bit for bit.
Q35_DEV float gdn_decay_dot8(float (&s)[16], const float* kk, float gt) {  // S *= g; this lane's part of S k
  float part[4];
#pragma unroll
  for (int pb = 0; pb < 4; ++pb) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = pb * 4 + i;
      s[e] = __fmul_rn(s[e], gt);
      acc = __fadd_rn(acc, __fmul_rn(s[e], kk[e]));
    }
    part[pb] = acc;
  }
  return __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
}
Q35_DEV float gdn_update_dot8(float (&s)[16], const float* kk, const float* qq, float delta) {  // S += k delta; part of S q
  float part[4];
#pragma unroll
  for (int pb = 0; pb < 4; ++pb) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = pb * 4 + i;
      s[e] = __fadd_rn(s[e], __fmul_rn(kk[e], delta));
      acc = __fadd_rn(acc, __fmul_rn(s[e], qq[e]));
    }
    part[pb] = acc;
  }
  return __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
}
// the row reduction: shuffle-xor 1, 2, 4
Q35_DEV float gdn_reduce8(float x) {
#pragma unroll
  for (int m = 1; m <= 4; m <<= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, m));
  return x;
}

// attention.metal:55-70 / the RoPE table: cos/sin of position * inv_freq for
// the 32 rotary pairs, evaluated in double from the f32 angle.
Q35_DEV void rope_pair(uint32_t position, int pair, float* cs) {
  const float arg = __fmul_rn(-__fmul_rn(float(pair), 0.03125f), 23.253496170043945f);
  const float inv_freq = (float)exp2((double)arg);
  const float angle = __fmul_rn(float(position), inv_freq);
  cs[2 * pair] = (float)cos((double)angle);
  cs[2 * pair + 1] = (float)sin((double)angle);
}

// Per-head RMSNorm (attention.metal:37-53: two 32-thread partials of 128
// values) followed by partial RoPE (attention.metal:55-70). One warp, one
// head; out[d] gets the bf16 value as f32.
Q35_DEV void head_norm_rope(const uint16_t* x, const uint16_t* gain,
                                               const float* cs, float* nrm, float* out, int lane) {
  // Lane l owns dims 4l..4l+3 and 128+4l..128+4l+3 (the reference's two
  // partial sums); every global load is issued up front. x, gain 8-byte
  // aligned, cs 16-byte aligned.
  const uint2 xa = *reinterpret_cast<const uint2*>(x + 4 * lane);
  const uint2 xb = *reinterpret_cast<const uint2*>(x + 128 + 4 * lane);
  const uint2 ga = *reinterpret_cast<const uint2*>(gain + 4 * lane);
  const uint2 gb = *reinterpret_cast<const uint2*>(gain + 128 + 4 * lane);
  float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = c0;  // (cos, sin) of pairs 4(l&7)..+3
  if (lane < 16) {
    c0 = reinterpret_cast<const float4*>(cs)[2 * (lane & 7)];
    c1 = reinterpret_cast<const float4*>(cs)[2 * (lane & 7) + 1];
  }
  const float va[4] = {bf_lo(xa.x), bf_hi(xa.x), bf_lo(xa.y), bf_hi(xa.y)};
  const float vb[4] = {bf_lo(xb.x), bf_hi(xb.x), bf_lo(xb.y), bf_hi(xb.y)};
  const float gA[4] = {bf_lo(ga.x), bf_hi(ga.x), bf_lo(ga.y), bf_hi(ga.y)};
  const float gB[4] = {bf_lo(gb.x), bf_hi(gb.x), bf_lo(gb.y), bf_hi(gb.y)};
  float pa = 0.0f, pb = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    pa = __fadd_rn(pa, __fmul_rn(va[i], va[i]));
    pb = __fadd_rn(pb, __fmul_rn(vb[i], vb[i]));
  }
  const float s0 = warp_sum(pa), s1 = warp_sum(pb);
  const float inv = drsqrtf(__fadd_rn(__fmul_rn(__fadd_rn(s0, s1), 0.00390625f), 1e-6f));
  float na[4], nb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    na[i] = bfr(__fmul_rn(bfr(__fmul_rn(va[i], inv)), gA[i]));
    nb[i] = bfr(__fmul_rn(bfr(__fmul_rn(vb[i], inv)), gB[i]));
  }
  *reinterpret_cast<float4*>(nrm + 4 * lane) = make_float4(na[0], na[1], na[2], na[3]);
  __syncwarp();
  if (lane < 16) {  // partial RoPE on dims 0..63: pair p = d & 31 rotates (p, p + 32)
    const float c[4] = {c0.x, c0.z, c1.x, c1.z}, sn[4] = {c0.y, c0.w, c1.y, c1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pair = 4 * (lane & 7) + i;
      const float lo = nrm[pair], hi = nrm[pair + 32];
      na[i] = lane < 8 ? bfr(__fsub_rn(__fmul_rn(lo, c[i]), __fmul_rn(hi, sn[i])))
                       : bfr(__fadd_rn(__fmul_rn(lo, sn[i]), __fmul_rn(hi, c[i])));
    }
  }
  *reinterpret_cast<float4*>(out + 4 * lane) = make_float4(na[0], na[1], na[2], na[3]);
  *reinterpret_cast<float4*>(out + 128 + 4 * lane) = make_float4(nb[0], nb[1], nb[2], nb[3]);
  __syncwarp();
}

// attention.metal:140-150: the attention output gate, sigmoid with BF16
// steps after exp, add and reciprocal (mirrored by sign).
Q35_DEV float attn_gate_bf(float x) {
  const float e = bfr(dexpf(fabsf(x)));
  const float denom = bfr(__fadd_rn(1.0f, e));
  const float inverse = bfr(__fdiv_rn(1.0f, denom));
  return bfr(x < 0.0f ? inverse : __fsub_rn(1.0f, inverse));
}

}  // namespace q35
