// Prompt chunks: the decode step's arithmetic for up to kPrefillTokens
// consecutive prompt tokens per launch.
//
// The reference consumes a prompt one row at a time through the same matvec
// and recurrence kernels as decode (rows = 1 path, model.rs:100-110). Here a
// chunk of tokens shares each launch: a matvec CTA streams its weight slice
// into shared memory once and applies it to every token of the chunk, and the
// recurrence keeps its state tile in registers across the chunk's tokens.
// Every token still goes through exactly the operations of the decode step,
// in the same order, so a prompt consumed in chunks leaves the same state,
// bit for bit, as one consumed token by token.
#include <cuda_runtime.h>

#include "q35_gdn.cuh"
#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_qmv.cuh"
#include "q35_types.h"

namespace q35 {

constexpr int kChunkThreads = 512;
constexpr int kChunkWarps = kChunkThreads / 32;
constexpr size_t kChunkSmemMax = 200 * 1024;

__host__ __device__ inline size_t chunk_align16(size_t v) { return (v + 15) & ~size_t(15); }

// Shared image of a chunk matvec CTA: its weight rows, the f32 activations of
// `sub` tokens in the lane-major layout the tasks read (token t, chunk c,
// group i, lane l -> float4 index (t * nch * 4 + c * 4 + i) * 32 + l; first
// the raw values, then the scaled x/16^j form), each lane's group-sum xs per
// (token, chunk), the row values of those tokens and the weight barrier.
struct ChunkLayout {
  size_t codes, scl, bia, xf, xs, vals, pl, bar, total;
};

// Rows of K >= 2048 (four or more 512-wide chunks) spread their chunks over
// warps and stage the per-lane chunk terms in shared memory (pl), summed in
// chunk order afterwards; shorter rows accumulate their chunks in registers.
__host__ __device__ inline bool chunk_split(int K) { return K >= 2048; }
__host__ __device__ inline ChunkLayout chunk_layout(int K, int rows, int sub) {
  ChunkLayout L;
  const int KW = K / 8, KG = K / 64;
  L.codes = 0;
  L.scl = L.codes + size_t(rows) * KW * 4;
  L.bia = L.scl + size_t(rows) * KG * 2;
  L.xf = chunk_align16(L.bia + size_t(rows) * KG * 2);
  L.xs = L.xf + size_t(sub) * K * 4;
  L.vals = L.xs + size_t(sub) * (K / 512) * 32 * 4;
  L.pl = chunk_align16(L.vals + size_t(sub) * rows * 4);
  const size_t pl_bytes = chunk_split(K) ? size_t(sub) * rows * (K / 512) * 32 * 4 : 0;
  L.bar = chunk_align16(L.pl + pl_bytes);
  L.total = L.bar + 16;
  return L;
}

__host__ __device__ inline int chunk_rows(const QmvArgs& a) {
  return a.epi == kEpiSwiglu ? 2 * a.units_per_cta : a.units_per_cta;
}

int chunk_sub_tokens(const QmvArgs& a) {
  int sub = a.ntok;
  while (sub > 1 && chunk_layout(a.K, chunk_rows(a), sub).total > kChunkSmemMax) --sub;
  return sub;
}

size_t chunk_smem_bytes(const QmvArgs& a) { return chunk_layout(a.K, chunk_rows(a), a.sub).total; }

// float4 slot of activation k of chunk token t in the lane-major layout
__device__ __forceinline__ int xf_slot(int t, int nch, int k) {
  const int c = k >> 9, l = (k & 511) >> 4, i = (k & 15) >> 2;
  return ((t * nch + c) * 4 + i) * 32 + l;
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(kChunkThreads, 1) k_qmv_chunk(const __grid_constant__ QmvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.K, KW = K / 8, KG = K / 64, nch = K / 512;
  Piece pc[4];
  const int np = qmv_pieces(a, blockIdx.x, pc);
  int nrows = 0;
  for (int i = 0; i < np; ++i) nrows += pc[i].count;
  const int rows_alloc = chunk_rows(a);
  const ChunkLayout L = chunk_layout(K, rows_alloc, a.sub);
  uint32_t* codes = reinterpret_cast<uint32_t*>(smem + L.codes);
  uint16_t* scl = reinterpret_cast<uint16_t*>(smem + L.scl);
  uint16_t* bia = reinterpret_cast<uint16_t*>(smem + L.bia);
  float4* xf = reinterpret_cast<float4*>(smem + L.xf);
  float* xsum = reinterpret_cast<float*>(smem + L.xs);
  float* vals = reinterpret_cast<float*>(smem + L.vals);
  float* pl = reinterpret_cast<float*>(smem + L.pl);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);

  // 1. Weights by bulk copy before the dependency wait (once for all tokens).
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0 && nrows > 0) {
    uint32_t bytes = 0;
    for (int i = 0; i < np; ++i) bytes += uint32_t(pc[i].count) * (KW * 4 + KG * 4);
    mbar_expect_tx(bar, bytes);
    int srow = 0;
    for (int i = 0; i < np; ++i) {
      const QmvSeg& sg = a.seg[pc[i].seg];
      const int n = pc[i].count;
      bulk_g2s(codes + size_t(srow) * KW, sg.w + size_t(pc[i].row0) * KW, uint32_t(n) * KW * 4, bar);
      bulk_g2s(scl + size_t(srow) * KG, sg.s + size_t(pc[i].row0) * KG, uint32_t(n) * KG * 2, bar);
      bulk_g2s(bia + size_t(srow) * KG, sg.b + size_t(pc[i].row0) * KG, uint32_t(n) * KG * 2, bar);
      srow += n;
    }
  }
  // epilogue row of this thread (thread i -> CTA row i)
  int e_seg = -1, e_row = 0;
  {
    int acc = 0;
    for (int p = 0; p < np; ++p) {
      if (tid >= acc && tid < acc + pc[p].count) {
        e_seg = pc[p].seg;
        e_row = pc[p].row0 + (tid - acc);
      }
      acc += pc[p].count;
    }
    if (EPI == kEpiSwiglu && tid >= pc[0].count) e_seg = -1;
  }
  // conv history and weights of this thread's channel (GDN input)
  uint16_t hh[3] = {0, 0, 0};
  uint16_t cw[4] = {0, 0, 0, 0};
  if (EPI == kEpiGdnConv && e_seg == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) cw[j] = a.convw[4 * e_row + j];
  }
  if (EPI == kEpiGdnConv && e_seg == 0 && !a.sess) {
    hh[0] = a.hist[e_row];
    hh[1] = a.hist[kGdnConv + e_row];
    hh[2] = a.hist[2 * kGdnConv + e_row];
  }

  pdl_wait();
  pdl_launch();
  uint32_t pos0 = 0;
  if (PRO == kProEmbedRms && a.sess) {
    // batched sessions: each session's step position and RoPE row
    if (blockIdx.x == 0)
      for (int i = tid; i < a.ntok * 32; i += kChunkThreads) {
        Ctl* c = a.ctls[i >> 5];
        const uint32_t p = ld_cg_u32(&c->pos);
        if ((i & 31) == 0) c->pos_step = p;
        rope_pair(p, i & 31, a.rope_out + 64 * (i >> 5));
      }
  } else if (PRO == kProEmbedRms) {
    pos0 = ld_cg_u32(&a.ctl->pos);
    if (blockIdx.x == 0) {
      if (tid == 0) a.ctl->pos_step = pos0;
      for (int i = tid; i < a.ntok * 32; i += kChunkThreads)
        rope_pair(pos0 + uint32_t(i >> 5), i & 31, a.rope_out + 64 * (i >> 5));
    }
  }

  const int ngroups = (nrows + 3) / 4;
  for (int t0 = 0; t0 < a.ntok; t0 += a.sub) {
    const int nt = min(a.sub, a.ntok - t0);
    // 2. Activations of the sub-chunk's tokens into the lane-major image.
    if (PRO == kProPlain) {
      const int per = K / 4;
      for (int idx = tid; idx < nt * per; idx += kChunkThreads) {
        const int t = idx / per, g4 = idx - t * per;
        xf[xf_slot(t, nch, 4 * g4)] = bf4(*reinterpret_cast<const uint2*>(a.x + size_t(t0 + t) * K + 4 * g4));
      }
    } else if (PRO == kProRms || PRO == kProEmbedRms) {
      for (int t = warp; t < nt; t += kChunkWarps) {
        float v[8][4];
        if (PRO == kProEmbedRms) {
          // linear.metal:19-23 for the token at position pos0 + t0 + t
          uint32_t token =
              a.sess ? ld_cg_u32(&a.seqs[t0 + t][ld_cg_u32(&a.ctls[t0 + t]->pos)])
                     : ld_cg_u32(&a.seq[pos0 + uint32_t(t0 + t)]);
          if (token >= uint32_t(kVocab)) {
            if (lane == 0) atomicCAS(&(a.sess ? a.ctls[t0 + t] : a.ctl)->err, 0u, kErrToken);
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
            if (blockIdx.x == 0) {
              uint2 hv;
              hv.x = pack_bf2(v[s][0], v[s][1]);
              hv.y = pack_bf2(v[s][2], v[s][3]);
              *reinterpret_cast<uint2*>(a.h_out + size_t(t0 + t) * kHidden + 128 * s + 4 * lane) = hv;
            }
          }
        } else {
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const float4 x4 = bf4(*reinterpret_cast<const uint2*>(a.x + size_t(t0 + t) * kHidden + 128 * s + 4 * lane));
            v[s][0] = x4.x, v[s][1] = x4.y, v[s][2] = x4.z, v[s][3] = x4.w;
          }
        }
        const float inv = rms1024_warp_inv(v);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const float4 g4 = bf4(*reinterpret_cast<const uint2*>(a.gain + 128 * s + 4 * lane));
          const float gn[4] = {g4.x, g4.y, g4.z, g4.w};
          float o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = bfr(__fmul_rn(bfr(__fmul_rn(v[s][j], inv)), gn[j]));
          xf[xf_slot(t, nch, 128 * s + 4 * lane)] = make_float4(o[0], o[1], o[2], o[3]);
        }
      }
    } else {  // kProNormGate: gdn.metal:238-254, one warp per (token, head)
      const float4 w4 = bf4(*reinterpret_cast<const uint2*>(a.gw + 4 * lane));
      const float w[4] = {w4.x, w4.y, w4.z, w4.w};
      for (int p = warp; p < nt * kGdnHeads; p += kChunkWarps) {
        const int t = p / kGdnHeads, hd = p - t * kGdnHeads;
        const size_t off = size_t(t0 + t) * 2048 + hd * 128 + 4 * lane;
        const float4 v4 = bf4(*reinterpret_cast<const uint2*>(a.gy + off));
        const float4 z4 = bf4(*reinterpret_cast<const uint2*>(a.gz + off));
        const float v[4] = {v4.x, v4.y, v4.z, v4.w}, z[4] = {z4.x, z4.y, z4.z, z4.w};
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = warp_sum(ss);
        const float inv = drsqrtf(__fadd_rn(__fmul_rn(ss, 0.0078125f), 1e-6f));
        float zg[4];
        if (a.gzs) {
          const float4 g4 = *reinterpret_cast<const float4*>(a.gzs + off);
          zg[0] = g4.x, zg[1] = g4.y, zg[2] = g4.z, zg[3] = g4.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) zg[i] = gdn_zgate(z[i]);
        }
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float norm = bfr(__fmul_rn(bfr(__fmul_rn(v[i], inv)), w[i]));
          o[i] = bfr(__fmul_rn(zg[i], norm));
        }
        xf[xf_slot(t, nch, hd * 128 + 4 * lane)] = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();
    // The decode step's per-lane constants of every (token, chunk): the
    // group sum xs = (((g0 + g1) + g2) + g3), g = ((x0 + x1) + x2) + x3 of the
    // lane's four groups, and the activations scaled to (x0, x1/16, x2/256,
    // x3/4096) in place.
    for (int idx = tid; idx < nt * nch * 32; idx += kChunkThreads) {
      const int t = idx / (nch * 32), rem = idx - t * nch * 32, c = rem >> 5, l = rem & 31;
      float g[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4& v = xf[((t * nch + c) * 4 + i) * 32 + l];
        const float4 x = v;
        g[i] = __fadd_rn(__fadd_rn(__fadd_rn(x.x, x.y), x.z), x.w);
        v = make_float4(x.x, __fmul_rn(x.y, 0.0625f), __fmul_rn(x.z, 0.00390625f),
                        __fmul_rn(x.w, 0.000244140625f));
      }
      xsum[idx] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, g[0]), g[1]), g[2]), g[3]);
    }
    __syncthreads();
    if (t0 == 0) mbar_wait(bar, 0, a.ctl, kErrQmvWait);

    // 3. Row terms per (group of four rows, block of kBlockTokens tokens),
    //    summed over the chunks in chunk order per lane, then the butterfly
    //    across lanes (reduce4): the decode step's finish.
    const int ntb = (nt + kBlockTokens - 1) / kBlockTokens;
    if (!chunk_split(K)) {
      for (int task = warp; task < ngroups * ntb; task += kChunkWarps) {
        const int g = task / ntb, j0 = (task - g * ntb) * kBlockTokens;
        const int nj = min(kBlockTokens, nt - j0);
        float acc[kBlockTokens][4];
#pragma unroll
        for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[j][r] = 0.0f;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          float term[kBlockTokens][4];
          qmv_block_terms(codes, scl, bia, nrows, 4 * g, c, KW, KG, nch, xf, xsum, j0, nj, lane, term);
#pragma unroll
          for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[j][r] = __fadd_rn(acc[j][r], term[j][r]);
        }
#pragma unroll
        for (int j = 0; j < kBlockTokens; ++j) {
          if (j < nj) {
            const float v = reduce4(acc[j][0], acc[j][1], acc[j][2], acc[j][3], lane);
            if ((lane & 7) == 0) {
              const int r = 4 * g + (((lane >> 4) & 1) << 1) + ((lane >> 3) & 1);
              if (r < nrows) vals[(j0 + j) * rows_alloc + r] = v;
            }
          }
        }
      }
    } else {
      // chunks over warps: per-lane terms to pl[((t * rows + row) * nch + c) * 32 + lane]
      for (int task = warp; task < ngroups * nch * ntb; task += kChunkWarps) {
        const int g = task / (nch * ntb), rem = task - g * nch * ntb;
        const int c = rem / ntb, j0 = (rem - c * ntb) * kBlockTokens;
        const int nj = min(kBlockTokens, nt - j0);
        float term[kBlockTokens][4];
        qmv_block_terms(codes, scl, bia, nrows, 4 * g, c, KW, KG, nch, xf, xsum, j0, nj, lane, term);
#pragma unroll
        for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r)
            if (j < nj && 4 * g + r < nrows)
              pl[((size_t(j0 + j) * rows_alloc + 4 * g + r) * nch + c) * 32 + lane] = term[j][r];
      }
      __syncthreads();
      for (int task = warp; task < ngroups * nt; task += kChunkWarps) {
        const int g = task / nt, t = task - g * nt;
        float p[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float acc = 0.0f;
          if (4 * g + r < nrows)
            for (int c = 0; c < nch; ++c)
              acc = __fadd_rn(acc, pl[((size_t(t) * rows_alloc + 4 * g + r) * nch + c) * 32 + lane]);
          p[r] = acc;
        }
        const float v = reduce4(p[0], p[1], p[2], p[3], lane);
        if ((lane & 7) == 0) {
          const int r = 4 * g + (((lane >> 4) & 1) << 1) + ((lane >> 3) & 1);
          if (r < nrows) vals[t * rows_alloc + r] = v;
        }
      }
    }
    __syncthreads();

    // 4. Epilogue, thread i finishes CTA row i for the sub-chunk's tokens in order.
    if (e_seg >= 0) {
      for (int t = 0; t < nt; ++t) {
        const size_t tt = size_t(t0 + t);
        const float v = vals[t * rows_alloc + tid];
        if (EPI == kEpiSwiglu) {
          const int n = pc[0].count;
          a.seg[0].y[tt * a.ystride[0] + pc[0].row0 + tid] =
              swiglu_bf(bfr(v), bfr(vals[t * rows_alloc + n + tid]));
        } else if (EPI == kEpiResAdd) {
          uint16_t* r = a.res + tt * kHidden + e_row;
          *r = f2bf(__fadd_rn(bf2f(*r), bfr(v)));
        } else if (EPI == kEpiGdnConv && e_seg == 0) {
          const uint16_t raw = f2bf(v);
          if (a.sess) {  // each session's own history
            uint16_t* hs = a.hists[tt] + a.hist_off;
            const uint16_t h0 = hs[e_row], h1 = hs[kGdnConv + e_row], h2 = hs[2 * kGdnConv + e_row];
            a.conv_out[tt * kGdnConv + e_row] = gdn_conv_value(h0, h1, h2, raw, cw);
            hs[e_row] = h1;
            hs[kGdnConv + e_row] = h2;
            hs[2 * kGdnConv + e_row] = raw;
          } else {
            a.conv_out[tt * kGdnConv + e_row] = gdn_conv_value(hh[0], hh[1], hh[2], raw, cw);
            hh[0] = hh[1];
            hh[1] = hh[2];
            hh[2] = raw;
          }
        } else {
          a.seg[e_seg].y[tt * a.ystride[e_seg] + e_row] = f2bf(v);
        }
      }
    }
    __syncthreads();
  }
  if (EPI == kEpiGdnConv && e_seg == 0 && !a.sess) {
    a.hist[e_row] = hh[0];
    a.hist[kGdnConv + e_row] = hh[1];
    a.hist[2 * kGdnConv + e_row] = hh[2];
  }
}

// GDN recurrence over a chunk's tokens (gdn.metal:176-228 with T > 1, as
// the reference loops over rows): grid (8 row blocks, 16 heads) x 64
// threads; the state tile stays in registers across tokens. The q/k norms
// and gates of all tokens are formed first, in parallel.
__global__ void __launch_bounds__(64) k_gdn_recur_chunk(const __grid_constant__ RecurArgs a) {
  __shared__ __align__(16) float st[16 * 128];
  __shared__ float qn[kPrefillTokens][128], kn[kPrefillTokens][128], gts[kPrefillTokens],
      bts[kPrefillTokens];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rb = blockIdx.x, h = blockIdx.y;
  const int nt = a.ntok;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, 16 * 128 * 4);
    bulk_g2s(st, a.state + (size_t(h) * 128 + rb * 16) * 128, 16 * 128 * 4, &bar);
  }
  const float e1 = dexpf(a.a_log[h]);
  const uint16_t dt = a.dt_bias[h];
  pdl_wait();
  pdl_launch();
  if (a.advance_pos && rb == 0 && h == 0 && tid == 0) a.ctl->pos = a.ctl->pos_step + uint32_t(nt);
  // warp 0 -> q, warp 1 -> k for every token; gates on lanes < nt
  for (int t = 0; t < nt; ++t)
    gdn_qk_norm(a.conv + size_t(t) * kGdnConv, h, warp == 0, lane, warp == 0 ? qn[t] : kn[t]);
  if (warp == 0 && lane < nt) gts[lane] = gdn_gate(a.a_raw[lane * 32 + h], dt, e1);
  if (warp == 1 && lane < nt) bts[lane] = gdn_beta(a.b_raw[lane * 32 + h]);
  if (a.zs)  // this CTA's 16 channels of every token
    for (int i = tid; i < nt * 16; i += 64) {
      const size_t off = size_t(i >> 4) * 2048 + h * 128 + rb * 16 + (i & 15);
      a.zs[off] = gdn_zgate(bf2f(a.z[off]));
    }
  __syncthreads();
  mbar_wait(&bar, 0, a.ctl, kErrRecurWait);
  const int row = tid >> 2, r = tid & 3;
  const int vrow = rb * 16 + row;
  float s[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = *reinterpret_cast<const float4*>(&st[row * 128 + r * 32 + i * 4]);
    s[i * 4 + 0] = t.x;
    s[i * 4 + 1] = t.y;
    s[i * 4 + 2] = t.z;
    s[i * 4 + 3] = t.w;
  }
  for (int t = 0; t < nt; ++t) {
    const float vv = bf2f(a.conv[size_t(t) * kGdnConv + 4096 + h * 128 + vrow]);
    const float out = gdn_row_step(s, kn[t] + r * 32, qn[t] + r * 32, gts[t], bts[t], vv);
    if (r == 0) a.y[size_t(t) * 2048 + h * 128 + vrow] = f2bf(out);
  }
  float4* dst = reinterpret_cast<float4*>(a.state + (size_t(h) * 128 + vrow) * 128 + r * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
}

// GDN recurrence for batched sessions: the decode step's k_gdn_recur for
// session blockIdx.z (its own state, conv row, gates and output row).
__global__ void __launch_bounds__(64) k_gdn_recur_sessions(const __grid_constant__ RecurArgs a) {
  __shared__ __align__(16) float st[16 * 128];
  __shared__ float qn[128], kn[128], gb[2];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rb = blockIdx.x, h = blockIdx.y, z = blockIdx.z;
  float* state = a.states[z] + a.state_off;
  const uint16_t* conv = a.conv + size_t(z) * kGdnConv;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, 16 * 128 * 4);
    bulk_g2s(st, state + (size_t(h) * 128 + rb * 16) * 128, 16 * 128 * 4, &bar);
  }
  pdl_wait();
  pdl_launch();
  Ctl* ctl = a.ctls[z];
  if (a.advance_pos && rb == 0 && h == 0 && tid == 0) ctl->pos = ctl->pos_step + 1;
  gdn_qk_norm(conv, h, warp == 0, lane, warp == 0 ? qn : kn);
  if (tid == 0) {
    gb[0] = gdn_gate(a.a_raw[z * 32 + h], a.dt_bias[h], dexpf(a.a_log[h]));
  } else if (tid == 32) {
    gb[1] = gdn_beta(a.b_raw[z * 32 + h]);
  }
  if (a.zs && tid >= 48) {  // this CTA's 16 channels of session z
    const size_t off = size_t(z) * 2048 + h * 128 + rb * 16 + (tid - 48);
    a.zs[off] = gdn_zgate(bf2f(a.z[off]));
  }
  __syncthreads();
  mbar_wait(&bar, 0, ctl, kErrRecurWait);
  const int row = tid >> 2, r = tid & 3;
  const int vrow = rb * 16 + row;
  float s[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = *reinterpret_cast<const float4*>(&st[row * 128 + r * 32 + i * 4]);
    s[i * 4 + 0] = t.x;
    s[i * 4 + 1] = t.y;
    s[i * 4 + 2] = t.z;
    s[i * 4 + 3] = t.w;
  }
  const float out = gdn_row_step(s, kn + r * 32, qn + r * 32, gb[0], gb[1], bf2f(conv[4096 + h * 128 + vrow]));
  if (r == 0) a.y[size_t(z) * 2048 + h * 128 + vrow] = f2bf(out);
  float4* dst = reinterpret_cast<float4*>(state + (size_t(h) * 128 + vrow) * 128 + r * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
#define Q35_CHUNK_VARIANTS(X)  \
  X(kProEmbedRms, kEpiGdnConv) \
  X(kProRms, kEpiGdnConv)      \
  X(kProRms, kEpiStore)        \
  X(kProRms, kEpiSwiglu)       \
  X(kProNormGate, kEpiResAdd)  \
  X(kProPlain, kEpiResAdd)

static void (*chunk_kernel(int pro, int epi))(QmvArgs) {
#define Q35_CHUNK_PICK(P, E) \
  if (pro == P && epi == E) return k_qmv_chunk<P, E>;
  Q35_CHUNK_VARIANTS(Q35_CHUNK_PICK)
#undef Q35_CHUNK_PICK
  return nullptr;
}

cudaError_t chunk_kernels_init() {
  cudaError_t e = cudaSuccess;
#define Q35_CHUNK_ATTR(P, E)                                                          \
  if (e == cudaSuccess)                                                               \
    e = cudaFuncSetAttribute(k_qmv_chunk<P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             int(kChunkSmemMax));
  Q35_CHUNK_VARIANTS(Q35_CHUNK_ATTR)
#undef Q35_CHUNK_ATTR
  return e;
}

cudaError_t launch_qmv_chunk(const QmvArgs& a, cudaStream_t st, bool pdl) {
  void (*kern)(QmvArgs) = chunk_kernel(a.pro, a.epi);
  if (!kern || a.ntok < 1 || a.ntok > kPrefillTokens || a.sub < 1) return cudaErrorInvalidValue;
  const int grid = (a.units + a.units_per_cta - 1) / a.units_per_cta;
  return launch_ex(kern, dim3(grid), dim3(kChunkThreads), chunk_smem_bytes(a), st, pdl, a);
}

cudaError_t launch_recur_sessions(const RecurArgs& a, int n, cudaStream_t st, bool pdl) {
  if (n < 1 || n > kMaxTensorSessions) return cudaErrorInvalidValue;
  return launch_ex(k_gdn_recur_sessions, dim3(8, kGdnHeads, n), dim3(64), 0, st, pdl, a);
}

cudaError_t launch_recur_chunk(const RecurArgs& a, cudaStream_t st, bool pdl) {
  if (a.ntok < 1 || a.ntok > kPrefillTokens) return cudaErrorInvalidValue;
  return launch_ex(k_gdn_recur_chunk, dim3(8, kGdnHeads), dim3(64), 0, st, pdl, a);
}

}  // namespace q35
