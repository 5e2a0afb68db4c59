// Q4 affine matvec building blocks (CUDA cores, batch 1), bit-exact with the
// reference's per-lane arithmetic.
//
// Layout is the MLX one the reference loads (weights.rs:50-52): codes
// [N][K/8] u32 with nibble k at bits 4*(k%8) of word k/8, scales and biases
// [N][K/64] bf16.
//
// Arithmetic (linear.metal:41-72): lane l of a SIMD group owns k = 512c +
// 16l .. +15 of every 512-wide chunk c. Per chunk it forms
//   xx = (x0, x1/16, x2/256, x3/4096, ...) and xs = sum of its 16 x values,
//   dotq = sum over the four 16-bit halves of ((t0 + t1) + t2) + t3 with
//   t_i = xx_i * float(half & (0xF << 4i)),
//   accum += s * dotq + xs * b,
// and the row value is the SIMD sum of the 32 accumulators (taken as an xor
// butterfly). Every product t_i is formed exactly as the reference rounds it
// without converting integers: the masked half-word OR'd into 0x4B000000 is
// the float 2^23 + m, and fmaf(2^23 + m, xx, -2^23 * xx) = round(m * xx) in
// one instruction. Products and sums are otherwise separately rounded
// (__fadd_rn / __fmul_rn), so the result equals the CPU restatement bit for
// bit.
#pragma once
#include "q35_dev.cuh"

namespace q35 {

constexpr float kTwo23 = 8388608.0f;

// Rows of a CTA of a fused matvec launch: CTA `cta` covers units
// [cta * upc, (cta + 1) * upc) of the concatenated segments (both the gate and
// the up row of each unit for SwiGLU), split into per-segment pieces.
struct Piece {
  int seg, row0, count;
};

__host__ __device__ inline int qmv_pieces(const QmvArgs& a, int cta, Piece* p) {
  const int u0 = cta * a.units_per_cta;
  const int u1 = (u0 + a.units_per_cta < a.units) ? u0 + a.units_per_cta : a.units;
  if (u1 <= u0) return 0;
  if (a.epi == kEpiSwiglu) {
    p[0] = {0, u0, u1 - u0};
    p[1] = {1, u0, u1 - u0};
    return 2;
  }
  int n = 0, off = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const int lo = u0 > off ? u0 : off;
    const int hi = u1 < off + a.seg[s].rows ? u1 : off + a.seg[s].rows;
    if (lo < hi) p[n++] = {s, lo - off, hi - lo};
    off += a.seg[s].rows;
  }
  return n;
}


// Per (chunk, lane) constants: xq[c][i][lane] float4 (i < 4: the 16 xx of
// the lane; the magic offsets -2^23 * xx are formed in registers, exactly,
// when loaded), xsum[c][lane] = the lane's xs. A thread
// builds one group of four consecutive k (one float4 of xx); the lane's xs
// is ((g0 + g1) + g2) + g3 over its four groups g = ((a + b) + c) + d, as the
// reference accumulates it. Dividing by 16/256/4096 is multiplying by the
// exact reciprocal powers of two (identical results). All threads must call.
Q35_DEV void build_xq(const float* xf, int K, float4* xq, float* xsum) {
  const int ngroups = K / 4;
  for (int base = 0; base < ngroups; base += blockDim.x) {
    const int t = base + threadIdx.x;
    const bool on = t < ngroups;
    float4 x4 = on ? *reinterpret_cast<const float4*>(xf + 4 * t) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float g = __fadd_rn(__fadd_rn(__fadd_rn(x4.x, x4.y), x4.z), x4.w);
    const float g1 = __shfl_down_sync(0xffffffffu, g, 1);
    const float g2 = __shfl_down_sync(0xffffffffu, g, 2);
    const float g3 = __shfl_down_sync(0xffffffffu, g, 3);
    if (on) {
      const int c = t >> 7, l = (t >> 2) & 31, j = t & 3;
      const float4 xx = make_float4(x4.x, __fmul_rn(x4.y, 0.0625f), __fmul_rn(x4.z, 0.00390625f),
                                    __fmul_rn(x4.w, 0.000244140625f));
      xq[(size_t(c) * 4 + j) * 32 + l] = xx;
      if (j == 0) xsum[c * 32 + l] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, g), g1), g2), g3);
    }
  }
}

// Emit the constants of one group of four consecutive activations
// (k = 4t .. 4t+3). The four groups of a lane (t = 4l' .. 4l'+3 within a
// chunk) must be held by four consecutive lanes of one warp in the same call;
// all lanes of the warp call (inactive ones with on = false).
Q35_DEV void emit_xq(int t, bool on, float4 x4, float4* xq, float* xsum) {
  const float g = __fadd_rn(__fadd_rn(__fadd_rn(x4.x, x4.y), x4.z), x4.w);
  const float g1 = __shfl_down_sync(0xffffffffu, g, 1);
  const float g2 = __shfl_down_sync(0xffffffffu, g, 2);
  const float g3 = __shfl_down_sync(0xffffffffu, g, 3);
  if (!on) return;
  const int c = t >> 7, l = (t >> 2) & 31, j = t & 3;
  const float4 xx = make_float4(x4.x, __fmul_rn(x4.y, 0.0625f), __fmul_rn(x4.z, 0.00390625f),
                                __fmul_rn(x4.w, 0.000244140625f));
  xq[(size_t(c) * 4 + j) * 32 + l] = xx;
  if (j == 0) xsum[c * 32 + l] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, g), g1), g2), g3);
}

Q35_DEV float4 bf4(uint2 u) { return make_float4(bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y)); }

Q35_DEV float magic(uint32_t bits) { return __uint_as_float(bits | 0x4b000000u); }

// ((t0 + t1) + t2) + t3 of one 16-bit half (low 16 bits of u). The four
// products are two packed fused multiply-adds (each component exactly the
// scalar fmaf) over consecutive k, whose xx and -2^23 xx already sit in
// register pairs.
Q35_DEV float half_dot(uint32_t u, const float4& xx, const float4& cc) {
  const float2 t01 = __ffma2_rn(make_float2(magic(u & 0x000fu), magic(u & 0x00f0u)), make_float2(xx.x, xx.y),
                                make_float2(cc.x, cc.y));
  const float2 t23 = __ffma2_rn(make_float2(magic(u & 0x0f00u), magic(u & 0xf000u)), make_float2(xx.z, xx.w),
                                make_float2(cc.z, cc.w));
  return __fadd_rn(__fadd_rn(__fadd_rn(t01.x, t01.y), t23.x), t23.y);
}

// The lane's chunk terms s*dotq + xs*b of rows [r0, r0+4) for chunk c (512
// wide), with the lane's chunk constants in registers; rows at or beyond
// nrows give 0.
Q35_DEV void qmv_rows_terms(const uint32_t* codes, const uint16_t* scl, const uint16_t* bia,
                            int nrows, int r0, int c, int K, const float4 (&xx)[4],
                            const float4 (&cc)[4], float xs, int lane, float (&term)[4]) {
  const int KW = K / 8, KG = K / 64;
  const int w0 = 64 * c + 2 * lane;
  const int g = 8 * c + (lane >> 2);
  uint2 q[4];
  float sc[4], bi[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = r0 + r < nrows ? r0 + r : nrows - 1;
    q[r] = *reinterpret_cast<const uint2*>(codes + size_t(row) * KW + w0);
    sc[r] = bf2f(scl[row * KG + g]);
    bi[r] = bf2f(bia[row * KG + g]);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float dotq = 0.0f;
    dotq = __fadd_rn(dotq, half_dot(q[r].x, xx[0], cc[0]));
    dotq = __fadd_rn(dotq, half_dot(q[r].x >> 16, xx[1], cc[1]));
    dotq = __fadd_rn(dotq, half_dot(q[r].y, xx[2], cc[2]));
    dotq = __fadd_rn(dotq, half_dot(q[r].y >> 16, xx[3], cc[3]));
    const float t = __fadd_rn(__fmul_rn(sc[r], dotq), __fmul_rn(xs, bi[r]));
    term[r] = r0 + r < nrows ? t : 0.0f;
  }
}

// One warp task with the lane's chunk constants in registers: rows
// [r0, r0+4) (those < nrows) of the CTA's smem image, chunk c (512 wide).
// Writes each lane's chunk term s*dotq + xs*b to pl[(row * nch + c) * 32 + lane].
Q35_DEV void qmv_chunk_core(const uint32_t* codes, const uint16_t* scl, const uint16_t* bia,
                            int nrows, int r0, int c, int K, const float4 (&xx)[4],
                            const float4 (&cc)[4], float xs, float* pl, int lane) {
  const int nch = K / 512;
  float term[4];
  qmv_rows_terms(codes, scl, bia, nrows, r0, c, K, xx, cc, xs, lane, term);
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (r0 + r < nrows) pl[(size_t(r0 + r) * nch + c) * 32 + lane] = term[r];
}

// The lane's constants of chunk c from the shared image built by build_xq.
Q35_DEV void load_xq(const float4* xq, const float* xsum, int c, int lane, float4 (&xx)[4],
                     float4 (&cc)[4], float& xs) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xx[i] = xq[(size_t(c) * 4 + i) * 32 + lane];
    cc[i] = make_float4(__fmul_rn(-kTwo23, xx[i].x), __fmul_rn(-kTwo23, xx[i].y),
                        __fmul_rn(-kTwo23, xx[i].z), __fmul_rn(-kTwo23, xx[i].w));
  }
  xs = xsum[c * 32 + lane];
}

// One warp task reading the chunk constants from shared memory.
Q35_DEV void qmv_chunk_task(const uint32_t* codes, const uint16_t* scl, const uint16_t* bia,
                            int nrows, int r0, int c, int K, const float4* xq, const float* xsum,
                            float* pl, int lane) {
  float4 xx[4], cc[4];
  float xs;
  load_xq(xq, xsum, c, lane, xx, cc, xs);
  qmv_chunk_core(codes, scl, bia, nrows, r0, c, K, xx, cc, xs, pl, lane);
}

// Tokens per warp task of the multi-token matvecs (prompt chunks, batched
// sessions, batched head): a task decodes its weight slice once and applies
// it to this many tokens.
constexpr int kBlockTokens = 4;

// Terms s*dot + xs*b of rows [r0, r0+4) (zero for rows >= nrows) for 512-wide
// chunk c and tokens j0 .. j0+nj-1 of a shared image holding, per token t,
// the scaled activations (x0, x1/16, x2/256, x3/4096) at float4
// ((t * nch + c) * 4 + i) * 32 + lane and the group sums at
// (t * nch + c) * 32 + lane (the layout build_xq writes per token). The lane's 16 nibbles
// of each row are decoded once into exact floats (the masked value n * 16^j,
// as the reference's pre-divided activations expect) and applied to every
// token. Each product n * x/16^j is exact, so fma(n, x, s) rounds exactly
// like the reference's s + n * x: the four-term sums, the lane's dot sum and
// s*dot + xs*b are the decode step's operations in the decode step's order.
Q35_DEV void qmv_block_terms(const uint32_t* codes, const uint16_t* scl,
                                                  const uint16_t* bia, int nrows, int r0, int c,
                                                  int KW, int KG, int nch, const float4* xf,
                                                  const float* xsum, int j0, int nj, int lane,
                                                  float (&term)[kBlockTokens][4]) {
  const int w0 = 64 * c + 2 * lane, gi = 8 * c + (lane >> 2);
  uint2 q[4];
  float sc[4], bi[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = r0 + r < nrows ? r0 + r : nrows - 1;
    q[r] = *reinterpret_cast<const uint2*>(codes + size_t(row) * KW + w0);
    sc[r] = bf2f(scl[row * KG + gi]);
    bi[r] = bf2f(bia[row * KG + gi]);
  }
#pragma unroll
  for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
    for (int r = 0; r < 4; ++r) term[j][r] = 0.0f;
#pragma unroll
  for (int hq = 0; hq < 4; ++hq) {
    float nv[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t u = ((hq < 2) ? q[r].x : q[r].y) >> (16 * (hq & 1));
      nv[r][0] = __fadd_rn(magic(u & 0x000fu), -kTwo23);
      nv[r][1] = __fadd_rn(magic(u & 0x00f0u), -kTwo23);
      nv[r][2] = __fadd_rn(magic(u & 0x0f00u), -kTwo23);
      nv[r][3] = __fadd_rn(magic(u & 0xf000u), -kTwo23);
    }
#pragma unroll
    for (int j = 0; j < kBlockTokens; ++j) {
      if (j < nj) {
        const float4 x = xf[(((j0 + j) * nch + c) * 4 + hq) * 32 + lane];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float h4 = __fmul_rn(nv[r][0], x.x);
          h4 = __fmaf_rn(nv[r][1], x.y, h4);
          h4 = __fmaf_rn(nv[r][2], x.z, h4);
          h4 = __fmaf_rn(nv[r][3], x.w, h4);
          term[j][r] = __fadd_rn(term[j][r], h4);  // the lane's dot sum
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kBlockTokens; ++j) {
    if (j < nj) {
      const float xs = xsum[((j0 + j) * nch + c) * 32 + lane];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float t = __fadd_rn(__fmul_rn(sc[r], term[j][r]), __fmul_rn(xs, bi[r]));
        term[j][r] = r0 + r < nrows ? t : 0.0f;
      }
    }
  }
}

// Transpose-reduce four per-lane values with the pairing of an xor butterfly
// (16, 8, 4, 2, 1): afterwards lanes 0, 8, 16, 24 hold the butterfly sums of
// rows 0, 1, 2, 3 (bit-identical to summing each row with a butterfly).
Q35_DEV float reduce4(float p0, float p1, float p2, float p3, int lane) {
  const bool h16 = lane & 16;
  float k0 = h16 ? p2 : p0, k1 = h16 ? p3 : p1;
  const float s0 = h16 ? p0 : p2, s1 = h16 ? p1 : p3;
  k0 = __fadd_rn(k0, __shfl_xor_sync(0xffffffffu, s0, 16));
  k1 = __fadd_rn(k1, __shfl_xor_sync(0xffffffffu, s1, 16));
  const bool h8 = lane & 8;
  float q = h8 ? k1 : k0;
  const float s = h8 ? k0 : k1;
  q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, s, 8));
  q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, 4));
  q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, 2));
  q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, 1));
  return q;
}

// Finish rows [r0, r0+4): accum = sum over chunks in order (linear.metal:41
// loop), then the SIMD sum. Writes vals[row].
Q35_DEV void qmv_finish_task(const float* pl, int nrows, int r0, int nch, float* vals, int lane) {
  float p[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float acc = 0.0f;
    if (r0 + r < nrows)
      for (int c = 0; c < nch; ++c) acc = __fadd_rn(acc, pl[(size_t(r0 + r) * nch + c) * 32 + lane]);
    p[r] = acc;
  }
  const float v = reduce4(p[0], p[1], p[2], p[3], lane);
  if ((lane & 7) == 0) {
    const int r = r0 + (((lane >> 4) & 1) << 1) + ((lane >> 3) & 1);
    if (r < nrows) vals[r] = v;
  }
}

// Block-level RMSNorm of a 1024-wide vector held as four contiguous values
// per thread (256 threads), in the reference's reduction order
// (linear_input_norm.metal:41-63): per-thread sequential sum of squares, SIMD
// butterfly, then a butterfly over the eight SIMD partials. Writes the bf16
// normalised value (as f32) to xf.
Q35_DEV void rms1024(const float v[4], const uint16_t* gain, float* xf, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc = __fadd_rn(acc, __fmul_rn(v[j], v[j]));
  acc = warp_sum(acc);
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  const float t0 = __fadd_rn(red[0], red[4]), t1 = __fadd_rn(red[1], red[5]);
  const float t2 = __fadd_rn(red[2], red[6]), t3 = __fadd_rn(red[3], red[7]);
  const float total = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
  const float inv = drsqrtf(__fadd_rn(__fmul_rn(total, 0.0009765625f), 1e-6f));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = 4 * tid + j;
    xf[c] = bfr(__fmul_rn(bfr(__fmul_rn(v[j], inv)), bf2f(gain[c])));
  }
}

// rms1024 for a block whose first 256 threads hold the vector (others pass
// zeros and ignore the result): normalised bf16 values returned in out[4].
Q35_DEV void rms1024_reg(const float v[4], const float g[4], float out[4], float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) acc = __fadd_rn(acc, __fmul_rn(v[j], v[j]));
  acc = warp_sum(acc);
  if (lane == 0 && warp < 8) red[warp] = acc;
  __syncthreads();
  const float t0 = __fadd_rn(red[0], red[4]), t1 = __fadd_rn(red[1], red[5]);
  const float t2 = __fadd_rn(red[2], red[6]), t3 = __fadd_rn(red[3], red[7]);
  const float total = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
  const float inv = drsqrtf(__fadd_rn(__fmul_rn(total, 0.0009765625f), 1e-6f));
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = bfr(__fmul_rn(bfr(__fmul_rn(v[j], inv)), g[j]));
}

// RMSNorm of one 1024-vector by one warp in the reference's block order
// (linear_input_norm.metal:41-63): lane l holds x[128 s + 4 l + j] in v[s][j],
// i.e. the four values of thread 32 s + l of a 256-thread block; each SIMD
// group's partial is that lane set's butterfly sum. Returns 1/rms.
Q35_DEV float rms1024_warp_inv(const float (&v)[8][4]) {
  float red[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = __fadd_rn(acc, __fmul_rn(v[s][j], v[s][j]));
    red[s] = warp_sum(acc);
  }
  const float t0 = __fadd_rn(red[0], red[4]), t1 = __fadd_rn(red[1], red[5]);
  const float t2 = __fadd_rn(red[2], red[6]), t3 = __fadd_rn(red[3], red[7]);
  const float total = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
  return drsqrtf(__fadd_rn(__fmul_rn(total, 0.0009765625f), 1e-6f));
}

}  // namespace q35
