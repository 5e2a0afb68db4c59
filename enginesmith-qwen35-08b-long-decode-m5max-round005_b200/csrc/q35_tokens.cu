// Per-token steps of the tensor-core routes: the operations between the GEMMs
// (q35_gemm.cu) for n tokens at once, token t = session t of a batched step
// or token t of a prompt chunk (q35_prompt.cu). Each is the decode step's
// arithmetic for that operation (the same device functions as the matvec
// prologues and epilogues), applied per token:
//   k_tok_rms      input RMSNorm (linear_input_norm.metal) of h[t]; in the
//                  first layer the token is embedded first (linear.metal:11-24)
//                  and its position and RoPE row recorded
//   k_tok_conv     GDN causal conv + SiLU and history shift (gdn_input.metal:163-177)
//   k_tok_normgate GDN gated RMS output (gdn.metal:238-254)
//   k_tok_swiglu   SwiGLU (linear_norm.metal:95-103)
#include <cuda_runtime.h>

#include "q35_gdn.cuh"
#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_qmv.cuh"
#include "q35_types.h"

namespace q35 {

// One warp per token.
__global__ void __launch_bounds__(32) k_tok_rms(const __grid_constant__ TokArgs a) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x, lane = threadIdx.x;
  float v[8][4];
  if (a.ew) {
    // batched sessions: session t's pending token at its position; prompt
    // chunk: token t of the session at p0 + t (token 0 moves the position past
    // the chunk; nothing in the chunk reads it)
    Ctl* c = a.seq ? a.ctl : a.ctls[t];
    uint32_t p;
    if (a.seq) {
      p = a.p0 + uint32_t(t);
      if (t == 0 && lane == 0) {
        c->pos_step = a.p0;
        c->pos = a.p0 + uint32_t(a.n);
      }
    } else {
      p = ld_cg_u32(&c->pos);
      if (lane == 0) c->pos_step = p;
    }
    rope_pair(p, lane, a.rope + 64 * t);
    uint32_t token = ld_cg_u32(a.seq ? &a.seq[p] : &a.seqs[t][p]);
    if (token >= uint32_t(kVocab)) {
      if (lane == 0) atomicCAS(&c->err, 0u, kErrToken);
      token = 0;
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const uint32_t word = a.ew[size_t(token) * (kHidden / 8) + 16 * s + (lane >> 1)];
      const int g = int(token) * (kHidden / 64) + 2 * s + (lane >> 4);
      const float sc = bf2f(a.es[g]), bs = bf2f(a.eb[g]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t q = (word >> (4 * (4 * (lane & 1) + j))) & 15u;
        v[s][j] = bfr(__fadd_rn(__fmul_rn(sc, float(q)), bs));
      }
      uint2 hv;
      hv.x = pack_bf2(v[s][0], v[s][1]);
      hv.y = pack_bf2(v[s][2], v[s][3]);
      *reinterpret_cast<uint2*>(a.h_out + size_t(t) * kHidden + 128 * s + 4 * lane) = hv;
    }
  } else {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const float4 x4 = bf4(*reinterpret_cast<const uint2*>(a.h_in + size_t(t) * kHidden + 128 * s + 4 * lane));
      v[s][0] = x4.x, v[s][1] = x4.y, v[s][2] = x4.z, v[s][3] = x4.w;
    }
  }
  const float inv = rms1024_warp_inv(v);
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const float4 g4 = bf4(*reinterpret_cast<const uint2*>(a.gain + 128 * s + 4 * lane));
    uint2 o;
    o.x = pack_bf2(bfr(__fmul_rn(bfr(__fmul_rn(v[s][0], inv)), g4.x)), bfr(__fmul_rn(bfr(__fmul_rn(v[s][1], inv)), g4.y)));
    o.y = pack_bf2(bfr(__fmul_rn(bfr(__fmul_rn(v[s][2], inv)), g4.z)), bfr(__fmul_rn(bfr(__fmul_rn(v[s][3], inv)), g4.w)));
    *reinterpret_cast<uint2*>(a.xn + size_t(t) * kHidden + 128 * s + 4 * lane) = o;
  }
}

// grid (kGdnConv / 256, n): channel c of token t through the session's history.
__global__ void __launch_bounds__(256) k_tok_conv(const __grid_constant__ TokArgs a) {
  pdl_wait();
  pdl_launch();
  const int c = blockIdx.x * 256 + threadIdx.x, t = blockIdx.y;
  uint16_t* hs = a.hists[t] + a.hist_off;
  const uint16_t raw = a.raw[size_t(t) * a.raw_stride + c];
  const uint16_t h0 = hs[c], h1 = hs[kGdnConv + c], h2 = hs[2 * kGdnConv + c];
  a.conv[size_t(t) * kGdnConv + c] = gdn_conv_value(h0, h1, h2, raw, a.convw + 4 * c);
  hs[c] = h1;
  hs[kGdnConv + c] = h2;
  hs[2 * kGdnConv + c] = raw;
}

// grid n, 16 warps: warp h normalises head h of token t and gates it.
__global__ void __launch_bounds__(512) k_tok_normgate(const __grid_constant__ TokArgs a) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x, lane = threadIdx.x & 31, hd = threadIdx.x >> 5;
  const size_t off = size_t(t) * 2048 + hd * 128 + 4 * lane;
  const float4 v4 = bf4(*reinterpret_cast<const uint2*>(a.y + off));
  const float4 w4 = bf4(*reinterpret_cast<const uint2*>(a.gw + 4 * lane));
  const float4 z4 = *reinterpret_cast<const float4*>(a.zs + off);
  const float v[4] = {v4.x, v4.y, v4.z, v4.w}, w[4] = {w4.x, w4.y, w4.z, w4.w};
  const float zg[4] = {z4.x, z4.y, z4.z, z4.w};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  ss = warp_sum(ss);
  const float inv = drsqrtf(__fadd_rn(__fmul_rn(ss, 0.0078125f), 1e-6f));
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = bfr(__fmul_rn(zg[i], bfr(__fmul_rn(bfr(__fmul_rn(v[i], inv)), w[i]))));
  uint2 r;
  r.x = pack_bf2(o[0], o[1]);
  r.y = pack_bf2(o[2], o[3]);
  *reinterpret_cast<uint2*>(a.gated + off) = r;
}

// grid (kMlp / 256, n)
__global__ void __launch_bounds__(256) k_tok_swiglu(const __grid_constant__ TokArgs a) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * 256 + threadIdx.x, t = blockIdx.y;
  const size_t o = size_t(t) * kMlp + i;
  a.act[o] = swiglu_bf(bf2f(a.g[o]), bf2f(a.u[o]));
}

cudaError_t launch_tok_rms(const TokArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_tok_rms, dim3(a.n), dim3(32), 0, st, pdl, a);
}
cudaError_t launch_tok_conv(const TokArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_tok_conv, dim3(kGdnConv / 256, a.n), dim3(256), 0, st, pdl, a);
}
cudaError_t launch_tok_normgate(const TokArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_tok_normgate, dim3(a.n), dim3(512), 0, st, pdl, a);
}
cudaError_t launch_tok_swiglu(const TokArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_tok_swiglu, dim3(kMlp / 256, a.n), dim3(256), 0, st, pdl, a);
}

}  // namespace q35
