// q35 decode kernels for sm_100a.
//
// One decode step (model.rs:228-307, rows == 1) is a chain of launches:
//   per GDN layer       : qmv[norm|qkv,z,a,b|conv] -> gdn_recur -> qmv[norm-gate|out|+res]
//   per attention layer : qmv[norm|q,k,v] -> attn (split-K, cluster combine, gate) -> qmv[o|+res]
//   per layer           : qmv[norm|gate,up|SwiGLU] -> qmv[down|+res]
//   once                : head (final norm, vocab projection, LSE, greedy)
// Every launch uses programmatic dependent launch: before griddepcontrol.wait
// a CTA only issues bulk copies of constant weights and of state written by
// earlier steps, so the next launch's weight stream overlaps this one's
// activation-dependent compute.
#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_qmv.cuh"
#include "q35_gdn.cuh"

namespace q35 {

// ---------------------------------------------------------------------------
// Q4 matvec with fused prologue / epilogue
// ---------------------------------------------------------------------------

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

struct QmvLayout {
  size_t codes, scl, bia, xq, xsum, xf, pl, vals, red, bar, total;
};
__host__ __device__ inline QmvLayout qmv_layout(int K, int rows) {
  QmvLayout L;
  const int KW = K / 8, KG = K / 64, nch = K / 512;
  L.codes = 0;
  L.scl = L.codes + size_t(rows) * KW * 4;
  L.bia = L.scl + size_t(rows) * KG * 2;
  L.xq = align16(L.bia + size_t(rows) * KG * 2);
  L.xsum = L.xq + size_t(nch) * 4 * 32 * 16;
  L.xf = L.xsum + size_t(nch) * 32 * 4;
  L.pl = L.xf + size_t(K) * 4;
  L.vals = L.pl + size_t(rows) * nch * 32 * 4;
  L.red = L.vals + size_t(rows) * 4;
  L.bar = align16(L.red + 64 * 4);
  L.total = L.bar + 16;
  return L;
}

size_t qmv_smem_bytes(const QmvArgs& a) {
  const int rows = a.epi == kEpiSwiglu ? 2 * a.units_per_cta : a.units_per_cta;
  return qmv_layout(a.K, rows).total;
}

// gdn_input.metal:419-431: 4-tap causal conv (tap 3 = current token), BF16
// boundary, SiLU with the BF16-stepped sigmoid, then the history shift.
__device__ __forceinline__ void gdn_conv_channel(int c, uint16_t raw, uint16_t* hist,
                                                 const uint16_t* convw, uint16_t* conv_out) {
  const uint16_t h0 = hist[c], h1 = hist[kGdnConv + c], h2 = hist[2 * kGdnConv + c];
  conv_out[c] = gdn_conv_value(h0, h1, h2, raw, convw + 4 * c);
  hist[c] = h1;
  hist[kGdnConv + c] = h2;
  hist[2 * kGdnConv + c] = raw;
}


__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr int kQmvThreads = 512;

// Specialised per (prologue, epilogue) pair at compile time, so a launch runs
// only its own code (smaller instruction footprint, no runtime branching on
// the variant); PRO and EPI must equal PRO and EPI.
template <int PRO, int EPI>
__global__ void __launch_bounds__(kQmvThreads, 1) k_qmv(const __grid_constant__ QmvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kQmvThreads / 32;
  const int K = a.K, KW = K / 8, KG = K / 64, nch = K / 512;
  // This CTA's rows per segment (cnt[s] rows from row r0[s] of segment s), in
  // registers: every loop over the four segments is unrolled with constant
  // indices (a dynamically indexed array lands in local memory, and the
  // parameter block read with a dynamic index; both cost a CTA that starts
  // as its predecessor ends most of a microsecond before it reaches the
  // dependency wait).
  int cnt[4], r0[4];
  {
    const int u0 = blockIdx.x * a.units_per_cta;
    const int u1 = min(u0 + a.units_per_cta, a.units);
#pragma unroll
    for (int sg = 0; sg < 4; ++sg) cnt[sg] = 0, r0[sg] = 0;
    if (EPI == kEpiSwiglu) {  // the gate rows, then the up rows, of the same units
      cnt[0] = cnt[1] = max(u1 - u0, 0);
      r0[0] = r0[1] = u0;
    } else {
      int off = 0;
#pragma unroll
      for (int sg = 0; sg < 4; ++sg) {
        if (sg < a.nseg) {
          const int rows = a.seg[sg].rows;
          const int lo = max(u0, off), hi = min(u1, off + rows);
          if (lo < hi) cnt[sg] = hi - lo, r0[sg] = lo - off;
          off += rows;
        }
      }
    }
  }
  const int nrows = cnt[0] + cnt[1] + cnt[2] + cnt[3];
  const int rows_alloc = EPI == kEpiSwiglu ? 2 * a.units_per_cta : a.units_per_cta;
  const QmvLayout L = qmv_layout(K, rows_alloc);
  uint32_t* codes = reinterpret_cast<uint32_t*>(smem + L.codes);
  uint16_t* scl = reinterpret_cast<uint16_t*>(smem + L.scl);
  uint16_t* bia = reinterpret_cast<uint16_t*>(smem + L.bia);
  float4* xq = reinterpret_cast<float4*>(smem + L.xq);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* pl = reinterpret_cast<float*>(smem + L.pl);
  float* vals = reinterpret_cast<float*>(smem + L.vals);
  float* red = reinterpret_cast<float*>(smem + L.red);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);

  // 1. Before the dependency wait: weights by bulk copy, and everything else
  //    written two or more launches back (gains, the residual, conv history).
  //    The last thread (which finishes no row at the model's shapes) sets up
  //    the barrier and issues the copies while the others preload; nobody
  //    waits on the barrier before the block barrier after the activations.
  constexpr int kIssuer = kQmvThreads - 1;
  if (tid == kIssuer) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (tid == kIssuer && nrows > 0) {
    mbar_expect_tx(bar, uint32_t(nrows) * (KW * 4 + KG * 4));
    int srow = 0;
#pragma unroll
    for (int sg = 0; sg < 4; ++sg) {
      const int n = cnt[sg];
      if (n > 0) {
        bulk_g2s(codes + size_t(srow) * KW, a.seg[sg].w + size_t(r0[sg]) * KW, uint32_t(n) * KW * 4, bar);
        bulk_g2s(scl + size_t(srow) * KG, a.seg[sg].s + size_t(r0[sg]) * KG, uint32_t(n) * KG * 2, bar);
        bulk_g2s(bia + size_t(srow) * KG, a.seg[sg].b + size_t(r0[sg]) * KG, uint32_t(n) * KG * 2, bar);
        srow += n;
      }
    }
  }
  // epilogue operands of the rows this thread finishes (thread i -> CTA row
  // i), loaded now and converted after the wait, so the loads stay in flight
  // meanwhile
  int e_seg = -1, e_row = 0;
  {
    int acc = 0;
#pragma unroll
    for (int sg = 0; sg < 4; ++sg) {
      if (tid >= acc && tid < acc + cnt[sg]) {
        e_seg = sg;
        e_row = r0[sg] + (tid - acc);
      }
      acc += cnt[sg];
    }
    if (EPI == kEpiSwiglu && tid >= cnt[0]) e_seg = -1;
  }
  uint16_t pre_res = 0, pre_h[3] = {0, 0, 0};
  uint2 pre_w4 = make_uint2(0u, 0u);
  if (e_seg >= 0) {
    if (EPI == kEpiResAdd) pre_res = a.res[e_row];
    if (EPI == kEpiGdnConv && e_seg == 0) {
      pre_h[0] = a.hist[e_row];
      pre_h[1] = a.hist[kGdnConv + e_row];
      pre_h[2] = a.hist[2 * kGdnConv + e_row];
      pre_w4 = *reinterpret_cast<const uint2*>(a.convw + 4 * e_row);
    }
  }
  uint2 gain_raw = make_uint2(0u, 0u);
  if ((PRO == kProRms || PRO == kProEmbedRms) && tid < 256) gain_raw = *reinterpret_cast<const uint2*>(a.gain + 4 * tid);

  // Norm-gate prologue: z (written two launches back) and the norm weight are
  // ready, so the gate factor z * sigmoid(z) of head `warp` is formed before
  // the wait; only the RMS of y waits for the recurrence.
  static_assert(kQmvThreads / 32 >= kGdnHeads, "one warp per GDN head");
  float ng_zs[4] = {0.f, 0.f, 0.f, 0.f}, ng_w[4] = {0.f, 0.f, 0.f, 0.f};
  if (PRO == kProNormGate && warp < kGdnHeads) {
    const float4 w4 = bf4(*reinterpret_cast<const uint2*>(a.gw + 4 * lane));
    ng_w[0] = w4.x, ng_w[1] = w4.y, ng_w[2] = w4.z, ng_w[3] = w4.w;
    if (a.gzs) {  // formed by the input projection's epilogue
      const float4 g4 = *reinterpret_cast<const float4*>(a.gzs + warp * 128 + 4 * lane);
      ng_zs[0] = g4.x, ng_zs[1] = g4.y, ng_zs[2] = g4.z, ng_zs[3] = g4.w;
    } else {
      const float4 z4 = bf4(*reinterpret_cast<const uint2*>(a.gz + warp * 128 + 4 * lane));
      ng_zs[0] = gdn_zgate(z4.x), ng_zs[1] = gdn_zgate(z4.y), ng_zs[2] = gdn_zgate(z4.z), ng_zs[3] = gdn_zgate(z4.w);
    }
  }

  // 2. Activations: every prologue leaves thread t with the group of four
  //    activations k = 4t .. 4t+3 and emits its matvec constants.
  // launch timing (the session's switch, written only by the host and by
  // launches that complete before this one starts): read before the wait
  const bool timing = a.ctl && ld_cg_u32(&a.ctl->timing_on);
  pdl_wait();
  pdl_launch();
  if (timing && tid == 0) atomicMin(&a.ctl->qmv_t0, globaltimer_ns());
  const float gain4[4] = {bf_lo(gain_raw.x), bf_hi(gain_raw.x), bf_lo(gain_raw.y), bf_hi(gain_raw.y)};
  if (PRO == kProPlain) {
    const int ngroups = K / 4;
    uint2 raw[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int t = it * kQmvThreads + tid;
      raw[it] = t < ngroups ? *reinterpret_cast<const uint2*>(a.x + 4 * t) : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int t = it * kQmvThreads + tid;
      if (it * kQmvThreads < ngroups) emit_xq(t, t < ngroups, bf4(raw[it]), xq, xsum);
    }
  } else if (PRO == kProRms || PRO == kProEmbedRms) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (PRO == kProEmbedRms) {
      // linear.metal:19-23 for the token the step consumes.
      const uint32_t pos = ld_cg_u32(&a.ctl->pos);
      uint32_t token = ld_cg_u32(&a.seq[pos]);
      if (token >= uint32_t(kVocab)) {
        if (tid == 0) atomicCAS(&a.ctl->err, 0u, kErrToken);
        token = 0;
      }
      if (tid < 256) {
        const uint32_t word = a.ew[size_t(token) * (kHidden / 8) + tid / 2];
        const int g = int(token) * (kHidden / 64) + (4 * tid) / 64;
        const float sc = bf2f(a.es[g]), bs = bf2f(a.eb[g]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = 4 * tid + j;
          const uint32_t q = (word >> (4 * (k % 8))) & 15u;
          v[j] = bfr(__fadd_rn(__fmul_rn(sc, float(q)), bs));
        }
        if (blockIdx.x == 0) {
#pragma unroll
          for (int j = 0; j < 4; ++j) a.h_out[4 * tid + j] = f2bf(v[j]);
        }
      }
      if (blockIdx.x == 0) {
        if (tid == 0) {
          a.ctl->pos_step = pos;
          a.ctl->token_step = token;
        }
        if (tid < 32) rope_pair(pos, tid, a.ctl->rope_cs);
      }
    } else if (tid < 256) {
      const float4 x4 = bf4(*reinterpret_cast<const uint2*>(a.x + 4 * tid));
      v[0] = x4.x;
      v[1] = x4.y;
      v[2] = x4.z;
      v[3] = x4.w;
    }
    float o[4];
    rms1024_reg(v, gain4, o, red);
    emit_xq(tid, tid < 256, make_float4(o[0], o[1], o[2], o[3]), xq, xsum);
  } else if (warp < kGdnHeads) {  // kProNormGate: gdn.metal:238-254, warp w -> head w
    const float4 v4 = bf4(*reinterpret_cast<const uint2*>(a.gy + warp * 128 + 4 * lane));
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    ss = warp_sum(ss);
    const float inv = drsqrtf(__fadd_rn(__fmul_rn(ss, 0.0078125f), 1e-6f));
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float norm = bfr(__fmul_rn(bfr(__fmul_rn(v[i], inv)), ng_w[i]));
      o[i] = bfr(__fmul_rn(ng_zs[i], norm));
    }
    emit_xq(warp * 32 + lane, true, make_float4(o[0], o[1], o[2], o[3]), xq, xsum);
  }
  __syncthreads();

  // 3. dot products from shared memory.
  mbar_wait(bar, 0, a.ctl, kErrQmvWait);
  const int ngroups = (nrows + 3) / 4;
  if (ngroups <= kWarps && nch <= (ngroups * nch + kWarps - 1) / kWarps) {
    // Whole groups: warp g walks the chunks of rows 4g..4g+3 in order and
    // keeps the lane's chunk sum in registers (the same additions, in chunk
    // order, as the shared-memory finish below), then the butterfly; taken
    // when the chunk tasks would need as many rounds anyway.
    if (warp < ngroups) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int c = 0; c < nch; ++c) {
        float4 xx[4], cc[4];
        float xs;
        load_xq(xq, xsum, c, lane, xx, cc, xs);
        float term[4];
        qmv_rows_terms(codes, scl, bia, nrows, 4 * warp, c, K, xx, cc, xs, lane, term);
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r] = __fadd_rn(acc[r], term[r]);
      }
      const float v = reduce4(acc[0], acc[1], acc[2], acc[3], lane);
      if ((lane & 7) == 0) {
        const int r = 4 * warp + (((lane >> 4) & 1) << 1) + ((lane >> 3) & 1);
        if (r < nrows) vals[r] = v;
      }
    }
    __syncthreads();
  } else {
    // a warp's tasks usually share their chunk: its constants are loaded once
    float4 xx[4], cc[4];
    float xs = 0.0f;
    int cur = -1;
    for (int task = warp; task < ngroups * nch; task += kWarps) {
      const int g = task / nch, c = task % nch;
      if (c != cur) {
        load_xq(xq, xsum, c, lane, xx, cc, xs);
        cur = c;
      }
      qmv_chunk_core(codes, scl, bia, nrows, 4 * g, c, K, xx, cc, xs, pl, lane);
    }
    __syncthreads();
    for (int g = warp; g < ngroups; g += kWarps) qmv_finish_task(pl, nrows, 4 * g, nch, vals, lane);
    __syncthreads();
  }

  // 4. epilogue (thread i finishes CTA row i).
  if (e_seg >= 0) {
    if (EPI == kEpiSwiglu) {
      a.seg[0].y[r0[0] + tid] = swiglu_bf(bfr(vals[tid]), bfr(vals[cnt[0] + tid]));
    } else {
      const float v = vals[tid];
      if (EPI == kEpiResAdd) {
        a.res[e_row] = f2bf(__fadd_rn(bf2f(pre_res), bfr(v)));
      } else if (EPI == kEpiGdnConv && e_seg == 0) {
        // gdn_input.metal:419-431
        const uint16_t raw = f2bf(v);
        float acc = 0.0f;
        acc = fmaf(bf2f(pre_h[0]), bf_lo(pre_w4.x), acc);
        acc = fmaf(bf2f(pre_h[1]), bf_hi(pre_w4.x), acc);
        acc = fmaf(bf2f(pre_h[2]), bf_lo(pre_w4.y), acc);
        acc = fmaf(bf2f(raw), bf_hi(pre_w4.y), acc);
        const float xq1 = bfr(acc);
        a.conv_out[e_row] = f2bf(__fmul_rn(xq1, sigmoid_bf(xq1)));
        a.hist[e_row] = pre_h[1];
        a.hist[kGdnConv + e_row] = pre_h[2];
        a.hist[2 * kGdnConv + e_row] = raw;
      } else {
        const uint16_t yb = f2bf(v);
        a.seg[e_seg].y[e_row] = yb;
        if (EPI == kEpiGdnConv && e_seg == 1 && a.zs_out) a.zs_out[e_row] = gdn_zgate(bf2f(yb));
      }
    }
  }
  // launch timing: the last CTA to finish closes the launch's interval and
  // adds its algorithmic bytes (rows x (K/2 code bytes + K/16 scale and bias bytes))
  if (timing) {
    __syncthreads();
    if (tid == 0) {
      atomicMax(&a.ctl->qmv_tend, globaltimer_ns());  // this CTA's end, before the accounting
      __threadfence();
      if (atomicAdd(&a.ctl->qmv_done, 1u) == gridDim.x - 1) {
        const unsigned long long t0 = atomicExch(&a.ctl->qmv_t0, ~0ull);
        const unsigned long long t1 = atomicExch(&a.ctl->qmv_tend, 0ull);
        atomicAdd(&a.ctl->qmv_ns, t1 - t0);
        unsigned long long rows = 0;
        for (int sg = 0; sg < a.nseg; ++sg) rows += unsigned(a.seg[sg].rows);
        atomicAdd(&a.ctl->qmv_bytes, rows * unsigned(K / 2 + K / 16));
        atomicAdd(&a.ctl->qmv_launches, 1u);
        atomicExch(&a.ctl->qmv_done, 0u);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// GDN recurrence (gdn.metal:176-228, T = 1) with the Q/K normalisation and
// gates of gdn_input.metal:433-460. Grid (8 row blocks, 16 heads) x 128
// threads: 8 lanes per value row, 16 f32 of state each, the reference's row
// reduction restated piecewise (gdn_decay_dot8 / gdn_reduce8 /
// gdn_update_dot8, bit-identical to gdn_row_step). After the dependency wait
// warps 0-3 form the q norm, the k norm, the decay gate and beta in parallel;
// exp(A_log), a weight, is formed before the wait.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) k_gdn_recur(const __grid_constant__ RecurArgs a) {
  __shared__ __align__(16) float st[16 * 128];
  __shared__ float qn[128], kn[128], gb[2];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rb = blockIdx.x, h = blockIdx.y;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, 16 * 128 * 4);
    bulk_g2s(st, a.state + (size_t(h) * 128 + rb * 16) * 128, 16 * 128 * 4, &bar);
  }
  const float e1 = warp == 2 && lane == 0 ? dexpf(a.a_log[h]) : 0.0f;
  pdl_wait();
  pdl_launch();
  if (a.advance_pos && rb == 0 && h == 0 && tid == 0) a.ctl->pos = a.ctl->pos_step + 1;
  // gdn_input.metal:433-441 (q, k) and :454-459 (g, beta)
  if (warp < 2) {
    gdn_qk_norm(a.conv, h, warp == 0, lane, warp == 0 ? qn : kn);
  } else if (lane == 0) {
    if (warp == 2) gb[0] = gdn_gate(a.a_raw[h], a.dt_bias[h], e1);
    else gb[1] = gdn_beta(a.b_raw[h]);
  }
  __syncthreads();
  mbar_wait(&bar, 0, a.ctl, kErrRecurWait);
  const int row = tid >> 3, r8 = tid & 7;
  const int vrow = rb * 16 + row;
  const float gt = gb[0], beta = gb[1];
  float s[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 t = *reinterpret_cast<const float4*>(&st[row * 128 + r8 * 16 + i * 4]);
    s[i * 4 + 0] = t.x;
    s[i * 4 + 1] = t.y;
    s[i * 4 + 2] = t.z;
    s[i * 4 + 3] = t.w;
  }
  const float memory = gdn_reduce8(gdn_decay_dot8(s, kn + r8 * 16, gt));
  const float delta = __fmul_rn(__fsub_rn(bf2f(a.conv[4096 + h * 128 + vrow]), memory), beta);
  const float out = gdn_reduce8(gdn_update_dot8(s, kn + r8 * 16, qn + r8 * 16, delta));
  if (r8 == 0) a.y[h * 128 + vrow] = f2bf(out);
  float4* dst = reinterpret_cast<float4*>(a.state + (size_t(h) * 128 + vrow) * 128 + r8 * 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
}

// Standalone conv/history step (the op-level GDN entry point; the decode
// step fuses the same channel function into the projection epilogue).
__global__ void k_gdn_conv(const uint16_t* raw, uint16_t* hist, const uint16_t* convw,
                           uint16_t* conv_out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < kGdnConv) gdn_conv_channel(c, raw[c], hist, convw, conv_out);
}

// ---------------------------------------------------------------------------
// GQA decode attention, bit-exact with the reference's two routes
// (attention_decode.metal):
//   len <  1024: sdpa_vector (:51-213): 32 chains per query head, chain g
//                visits keys g, g+32, ...; f32 partials, then the in-group
//                combine (:194-212) and attn_gate (attention.metal:133-151);
//   len >= 1024: sdpa_vector_2pass_1 (:215-431): 64 chains, chain b visits
//                keys b, b+64, ...; bf16 unnormalised partials, then
//                attn_decode_split2_gate (:830-891).
// Each chain is an online softmax over its keys in order:
//   m' = max(m, s); f = exp(m - m'); e = exp(s - m'); S = S*f + e;
//   o = o*f + e*v.
// One CTA owns one chain for the four query heads of a kv head, so every
// K/V row is read once. Rows stream through a ring of bulk copies. Scores use
// the reference's per-lane order (eight products per lane, then a SIMD sum);
// the running max is a prefix scan and f, e are independent, so only the S/o
// recurrence runs key by key. k_attn_combine then combines the chains and
// applies the BF16 output gate.
// ---------------------------------------------------------------------------
struct AttnSmem {
  uint16_t kt[kAttnStages][kAttnTile][kHeadDim];  // K ring
  uint16_t vt[kAttnStages][kAttnTile][kHeadDim];  // V ring
  float q[4][kHeadDim];
  float nrm[5][kHeadDim];
  float kr[kHeadDim];
  uint16_t kf[kHeadDim], vf[kHeadDim];
  float sc[kAttnBufs][4][kAttnTile];  // scores [buffer][head][key]
  float4 f[kAttnBufs][kAttnTile];     // per key: the four heads' factors
  float4 e[kAttnBufs][kAttnTile];     // per key: the four heads' weights
  uint32_t fm[kAttnBufs][4];          // per head: keys whose factor is not 1
  uint64_t kfull[kAttnStages], kempty[kAttnStages], vfull[kAttnStages], vempty[kAttnStages];
  uint64_t scfull[kAttnBufs], scempty[kAttnBufs], fefull[kAttnBufs], feempty[kAttnBufs];
};

size_t attn_smem_bytes() { return sizeof(AttnSmem); }

// Butterfly-order transpose reduction of 16 per-lane values: afterwards lane
// L (and L^1) holds the sum of value (L >> 1).
__device__ __forceinline__ float reduce16(float* v, int lane) {
#pragma unroll
  for (int m = 16, h = 8; m >= 2; m >>= 1, h >>= 1) {
    const bool hi = lane & m;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float keep = hi ? v[i + h] : v[i];
      const float send = hi ? v[i] : v[i + h];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
    }
  }
  return __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
}

// Launch timing: the earliest post-dependency start over CTAs to the latest
// CTA end (taken before the accounting atomics, whose round trips are not
// part of the launch's work), accumulated in the control block when enabled.
__device__ __forceinline__ void attn_time_start(Ctl* ctl, bool timing) {
  if (timing) atomicMin(&ctl->attn_t0, globaltimer_ns());
}
__device__ __forceinline__ void attn_time_end(Ctl* ctl, bool timing) {
  if (!timing) return;
  atomicMax(&ctl->attn_tend, globaltimer_ns());  // this CTA's end, before the accounting
  __threadfence();
  if (atomicAdd(&ctl->attn_done, 1u) == gridDim.x * gridDim.y - 1) {
    const unsigned long long t0 = atomicExch(&ctl->attn_t0, ~0ull);
    const unsigned long long t1 = atomicExch(&ctl->attn_tend, 0ull);
    atomicAdd(&ctl->attn_ns, t1 - t0);
    atomicAdd(&ctl->attn_launches, 1u);
    atomicExch(&ctl->attn_done, 0u);
  }
}


// Warp roles, linked only by full/empty mbarrier pairs (every wait bounded):
//   warps 0-7   score: keys 4w..4w+3 of each tile for the four query heads
//   warps 8-11  scan: one query head each; running max as a prefix scan,
//               then the factors f and weights e of the tile's keys
//   warps 12-15 recurrence: lane l of warp r owns dims 64r + 2l, +1 of all
//               four heads, so each V element is unpacked once for 4 heads
//   warp 16     K producer, warp 17 V producer (one bulk copy per tile)
// The current token's key/value (written to the cache by this kernel) are
// read from their staging copies kf/vf, never from the ring.
constexpr int kAttnScoreWarps = 8, kAttnScanWarp0 = 8, kAttnRecWarp0 = 12;
constexpr int kAttnKProdWarp = 16, kAttnVProdWarp = 17;

// Session z's view of a batched launch's arguments.
__device__ __forceinline__ AttnArgs attn_session_view(const AttnArgs& a, int z) {
  AttnArgs v = a;
  const AttnSess& ss = a.sess[z];
  v.kcache = ss.kcache;
  v.vcache = ss.vcache;
  v.capacity = ss.capacity;
  v.ctl = ss.ctl;
  v.q_raw = a.q_raw + size_t(z) * kQProj;
  v.k_raw = a.k_raw + size_t(z) * kKvHeads * kHeadDim;
  v.v_raw = a.v_raw + size_t(z) * kKvHeads * kHeadDim;
  v.gated = a.gated + size_t(z) * kQHeads * kHeadDim;
  v.rope = a.rope + 64 * z;
  v.part_o = a.part_o + size_t(z) * kKvHeads * kAttnChains * 4 * kHeadDim;
  v.part_ml = a.part_ml + size_t(z) * kKvHeads * kAttnChains * 4 * 2;
  return v;
}

template <bool SESS>
__global__ void __launch_bounds__(kAttnThreads, 1) k_attn(const __grid_constant__ AttnArgs a_in) {
  AttnArgs sv;
  if constexpr (SESS) sv = attn_session_view(a_in, blockIdx.z);
  const AttnArgs& a = SESS ? sv : a_in;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chain = blockIdx.x, kh = blockIdx.y;
  const uint32_t cap = a.capacity;
  constexpr float kMin = -3.4028234663852886e38f;

  // pos_step was written by the step's first launch (>= 2 launches back);
  // a prompt chunk's token t sits pos_add = t places after it.
  const uint32_t pos = ld_cg_u32(&a.ctl->pos_step) + uint32_t(a.pos_add);
  // sequence split: the local keys are positions r, r + G, ... <= pos; the
  // current token is local (at local index len - 1) on rank pos % G only
  const bool xs = a.xworld > 1;
  const uint32_t xg = xs ? uint32_t(a.xworld) : 1u, xr = xs ? uint32_t(a.xrank) : 0u;
  const uint32_t len = xs ? (pos >= xr ? (pos - xr) / xg + 1 : 0u) : pos + 1;
  const bool mine = !xs || pos % xg == xr;
  const uint32_t lpos = mine ? len - 1 : 0u;
  const float* rope = a.rope ? a.rope : a.ctl->rope_cs;
  const bool split = xs || len >= 1024;
  const int stride = split ? 64 : 32;
  const int nkeys = (chain < stride && uint32_t(chain) < len) ? int((len - 1 - chain) / stride) + 1 : 0;
  const int ntiles = (nkeys + kAttnTile - 1) / kAttnTile;
  // Chain-major cache: position p at chain p % 64, slot p / 64. A split-route
  // tile is one contiguous run of a chain; a short-route chain (stride 32)
  // interleaves chains c and c + 32, loaded as two runs into rows 0-15 / 16-31.
  const size_t cps = cap / kAttnChains;
  const uint16_t* kbase = a.kcache + size_t(kh) * cap * kHeadDim;
  const uint16_t* vbase = a.vcache + size_t(kh) * cap * kHeadDim;
  auto row_of = [&](int j) { return split ? j : ((j & 1) << 4) + (j >> 1); };
  // the current token is key `pos`: chain pos % stride, local index pos / stride
  // (the chain's last key)
  const bool owner = mine && chain == int(lpos % stride);
  const int own_idx = int(lpos / stride);
  const int own_t = owner ? own_idx / kAttnTile : -1, own_j = own_idx % kAttnTile;

  auto issue = [&](const uint16_t* base, uint16_t (*ring)[kHeadDim], uint64_t* bar, int t) {
    const int n = min(kAttnTile, nkeys - t * kAttnTile);
    mbar_expect_tx(bar, uint32_t(n) * kHeadDim * 2);
    if (split) {
      const size_t off = (size_t(chain) * cps + size_t(t) * kAttnTile) * kHeadDim;
      bulk_g2s(&ring[0][0], base + off, uint32_t(n) * kHeadDim * 2, bar);
    } else {
      const int na = (n + 1) >> 1, nb = n >> 1;
      bulk_g2s(&ring[0][0], base + size_t(chain) * cps * kHeadDim, uint32_t(na) * kHeadDim * 2, bar);
      if (nb > 0)
        bulk_g2s(&ring[16][0], base + size_t(chain + 32) * cps * kHeadDim, uint32_t(nb) * kHeadDim * 2,
                 bar);
    }
  };
  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&S.kfull[s], 1);
      mbar_init(&S.kempty[s], kAttnScoreWarps);
      mbar_init(&S.vfull[s], 1);
      mbar_init(&S.vempty[s], 4);
    }
    for (int b = 0; b < kAttnBufs; ++b) {
      mbar_init(&S.scfull[b], kAttnScoreWarps);
      mbar_init(&S.scempty[b], 4);
      mbar_init(&S.fefull[b], 4);
      mbar_init(&S.feempty[b], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const bool kprod = warp == kAttnKProdWarp && lane == 0, vprod = warp == kAttnVProdWarp && lane == 0;
  if (kprod)
    for (int t = 0; t < kAttnStages && t < ntiles; ++t) issue(kbase, S.kt[t], &S.kfull[t], t);
  if (vprod)
    for (int t = 0; t < kAttnStages && t < ntiles; ++t) issue(vbase, S.vt[t], &S.vfull[t], t);
  const bool timing = ld_cg_u32(&a.ctl->timing_on);  // read before the wait (host-set switch)
  pdl_wait();
  pdl_launch();
  if (tid == 0) attn_time_start(a.ctl, timing);

  // Query heads 4kh..4kh+3 (warps 0-3) scaled by 1/16 (attention_decode.metal:289);
  // warp 4 prepares the current token's key (attention.metal:295-311).
  if (warp < 4) {
    const int qh = 4 * kh + warp;
    head_norm_rope(a.q_raw + qh * 512, a.q_gain, rope, S.nrm[warp], S.q[warp], lane);
    for (int d = lane; d < kHeadDim; d += 32) S.q[warp][d] = __fmul_rn(0.0625f, S.q[warp][d]);
  } else if (warp == 4) {
    const uint4 vr = *reinterpret_cast<const uint4*>(a.v_raw + kh * kHeadDim + 8 * lane);
    head_norm_rope(a.k_raw + kh * kHeadDim, a.k_gain, rope, S.nrm[4], S.kr, lane);
    const float* kr8 = S.kr + 8 * lane;
    const uint4 kb = make_uint4(pack_bf2(kr8[0], kr8[1]), pack_bf2(kr8[2], kr8[3]),
                                pack_bf2(kr8[4], kr8[5]), pack_bf2(kr8[6], kr8[7]));
    *reinterpret_cast<uint4*>(S.kf + 8 * lane) = kb;
    *reinterpret_cast<uint4*>(S.vf + 8 * lane) = vr;
    if (owner) {
      const size_t ci = (size_t(kh) * cap + size_t(lpos % kAttnChains) * cps + lpos / kAttnChains) * kHeadDim;
      *reinterpret_cast<uint4*>(a.kcache + ci + 8 * lane) = kb;
      *reinterpret_cast<uint4*>(a.vcache + ci + 8 * lane) = vr;
    }
    __syncwarp();
  }
  __syncthreads();

  const size_t pbase = (size_t(kh) * kAttnChains + chain) * 4;  // + head
  if (warp < kAttnScoreWarps) {
    // ---------------- score warps ----------------
    // lane l owns dims 8l..8l+7 of every head (as the reference).
    // Heads (0,1) and (2,3) share packed f32x2 products and adds, so each
    // score keeps the scalar sequence of rounded products and sums: the adds
    // are __fadd2_rn (each component as __fadd_rn), the products prod2 (each
    // component exactly the rounded product). A packed multiply is not used:
    // ptxas (CUDA 12.9, sm_100a) fuses it into the packed add that consumes
    // it, even with explicit .rn on both and under -fmad=false (measured).
    const float2 nzs = make_float2(a.nzero, a.nzero);
    float2 qp[2][8];
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int e = 0; e < 8; ++e) qp[p][e] = make_float2(S.q[2 * p][8 * lane + e], S.q[2 * p + 1][8 * lane + e]);
    for (int t = 0; t < ntiles; ++t) {
      const int st = t % kAttnStages, sb = t % kAttnBufs;
      mbar_wait(&S.kfull[st], uint32_t(t / kAttnStages) & 1u, a.ctl, kErrAttnWait);
      float v[16];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * warp + jj;
        const uint16_t* krow = (t == own_t && j == own_j) ? S.kf : S.kt[st][row_of(j)];
        const uint4 kv = *reinterpret_cast<const uint4*>(krow + 8 * lane);
        const float k8[8] = {bf_lo(kv.x), bf_hi(kv.x), bf_lo(kv.y), bf_hi(kv.y),
                             bf_lo(kv.z), bf_hi(kv.z), bf_lo(kv.w), bf_hi(kv.w)};
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          float2 sc = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int e = 0; e < 8; ++e) sc = __fadd2_rn(sc, prod2(qp[p][e], make_float2(k8[e], k8[e]), nzs));
          v[(2 * p) * 4 + jj] = sc.x;
          v[(2 * p + 1) * 4 + jj] = sc.y;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.kempty[st]);
      const float r = reduce16(v, lane);
      if (t >= kAttnBufs)
        mbar_wait(&S.scempty[sb], uint32_t(t / kAttnBufs - 1) & 1u, a.ctl, kErrAttnWait);
      if ((lane & 1) == 0) S.sc[sb][lane >> 3][4 * warp + ((lane >> 1) & 3)] = r;
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.scfull[sb]);
    }
  } else if (warp < kAttnRecWarp0) {
    // ---------------- scan warps ----------------
    const int h = warp - kAttnScanWarp0;
    float msum = kMin;  // running max of head h
    for (int t = 0; t < ntiles; ++t) {
      const int sb = t % kAttnBufs;
      const int nk = min(kAttnTile, nkeys - t * kAttnTile);
      mbar_wait(&S.scfull[sb], uint32_t(t / kAttnBufs) & 1u, a.ctl, kErrAttnWait);
      const float sv = lane < nk ? S.sc[sb][h][lane] : -INFINITY;
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.scempty[sb]);
      float v = sv;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v = fmaxf(v, u);
      }
      const float mt = fmaxf(msum, v);
      float mprev = __shfl_up_sync(0xffffffffu, mt, 1);
      if (lane == 0) mprev = msum;
      const float fj = fexp(__fsub_rn(mprev, mt)), ej = fexp(__fsub_rn(sv, mt));
      const uint32_t fm = __ballot_sync(0xffffffffu, lane < nk && fj != 1.0f);
      msum = __shfl_sync(0xffffffffu, mt, nk - 1);
      if (t >= kAttnBufs)
        mbar_wait(&S.feempty[sb], uint32_t(t / kAttnBufs - 1) & 1u, a.ctl, kErrAttnWait);
      reinterpret_cast<float*>(&S.f[sb][lane])[h] = fj;
      reinterpret_cast<float*>(&S.e[sb][lane])[h] = ej;
      if (lane == 0) S.fm[sb][h] = fm;
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.fefull[sb]);
    }
    if (lane == 0) a.part_ml[(pbase + h) * 2] = msum;
  } else if (warp < kAttnKProdWarp) {
    // ---------------- recurrence warps ----------------
    const int wr = warp - kAttnRecWarp0, d = 64 * wr + 2 * lane, hs = lane & 3;
    // o2[i][p] = (o of head 2p, o of head 2p+1) at dim d + i. Products are
    // packed prod2 (the rounded products, never fused with the add); the adds
    // are packed __fadd2_rn.
    float2 o2[2][2] = {{{0.0f, 0.0f}, {0.0f, 0.0f}}, {{0.0f, 0.0f}, {0.0f, 0.0f}}};
    float ssum = 0.0f;  // running sum of head lane & 3
    const float2 nz2 = make_float2(a.nzero, a.nzero);
    for (int t = 0; t < ntiles; ++t) {
      const int st = t % kAttnStages, b = t % kAttnBufs;
      const int nk = min(kAttnTile, nkeys - t * kAttnTile);
      mbar_wait(&S.fefull[b], uint32_t(t / kAttnBufs) & 1u, a.ctl, kErrAttnWait);
      mbar_wait(&S.vfull[st], uint32_t(t / kAttnStages) & 1u, a.ctl, kErrAttnWait);
      const uint32_t fm = S.fm[b][0] | S.fm[b][1] | S.fm[b][2] | S.fm[b][3];
      // S = S*f + e, o = o*f + e*v key by key (attention_decode.metal:357-366);
      // keys whose four factors are all 1 skip the (exact) multiply by 1.
#define Q35_ATTN_ACC(J, VV)                                                    \
  {                                                                            \
    const float4 e4 = S.e[b][J];                                               \
    const float es = reinterpret_cast<const float*>(&S.e[b][J])[hs];           \
    const float v0 = bf_lo(VV), v1 = bf_hi(VV);                                \
    const float2 e01 = make_float2(e4.x, e4.y), e23 = make_float2(e4.z, e4.w); \
    ssum = __fadd_rn(ssum, es);                                                \
    o2[0][0] = __fadd2_rn(o2[0][0], prod2(e01, make_float2(v0, v0), nz2)); \
    o2[0][1] = __fadd2_rn(o2[0][1], prod2(e23, make_float2(v0, v0), nz2)); \
    o2[1][0] = __fadd2_rn(o2[1][0], prod2(e01, make_float2(v1, v1), nz2)); \
    o2[1][1] = __fadd2_rn(o2[1][1], prod2(e23, make_float2(v1, v1), nz2)); \
  }
#define Q35_ATTN_RESCALE(J)                                                    \
  {                                                                            \
    const float4 f4 = S.f[b][J];                                               \
    ssum = __fmul_rn(ssum, reinterpret_cast<const float*>(&S.f[b][J])[hs]);    \
    o2[0][0] = prod2(o2[0][0], make_float2(f4.x, f4.y), nz2); \
    o2[0][1] = prod2(o2[0][1], make_float2(f4.z, f4.w), nz2); \
    o2[1][0] = prod2(o2[1][0], make_float2(f4.x, f4.y), nz2); \
    o2[1][1] = prod2(o2[1][1], make_float2(f4.z, f4.w), nz2); \
  }
      if (split && t != own_t) {
        if (fm == 0) {
#pragma unroll 8
          for (int j = 0; j < nk; ++j) {
            const uint32_t vv = *reinterpret_cast<const uint32_t*>(&S.vt[st][j][d]);
            Q35_ATTN_ACC(j, vv)
          }
        } else {  // some factor differs from 1: multiply every key (x * 1 == x)
#pragma unroll 8
          for (int j = 0; j < nk; ++j) {
            const uint32_t vv = *reinterpret_cast<const uint32_t*>(&S.vt[st][j][d]);
            Q35_ATTN_RESCALE(j)
            Q35_ATTN_ACC(j, vv)
          }
        }
      } else {
        for (int j = 0; j < nk; ++j) {
          if ((fm >> j) & 1u) Q35_ATTN_RESCALE(j)
          const uint16_t* vrow = (t == own_t && j == own_j) ? S.vf : S.vt[st][row_of(j)];
          const uint32_t vv = *reinterpret_cast<const uint32_t*>(vrow + d);
          Q35_ATTN_ACC(j, vv)
        }
      }
#undef Q35_ATTN_RESCALE
#undef Q35_ATTN_ACC
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.vempty[st]);
        mbar_arrive(&S.feempty[b]);
      }
    }
    // chain partials (bf16-rounded on the split route, attention_decode.metal:428-430;
    // kept in f32 under a sequence split, whose rank merge has no reference form)
    const bool round_part = split && !xs;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float oa = (h & 1) ? o2[0][h >> 1].y : o2[0][h >> 1].x;
      const float ob = (h & 1) ? o2[1][h >> 1].y : o2[1][h >> 1].x;
      float* po = a.part_o + (pbase + h) * kHeadDim + d;
      po[0] = round_part ? bfr(oa) : oa;
      po[1] = round_part ? bfr(ob) : ob;
    }
    if (wr == 0 && lane < 4) a.part_ml[(pbase + lane) * 2 + 1] = ssum;
  } else if (kprod) {
    // ---------------- K producer ----------------
    for (int t = kAttnStages; t < ntiles; ++t) {
      const int st = t % kAttnStages;
      mbar_wait(&S.kempty[st], uint32_t(t / kAttnStages - 1) & 1u, a.ctl, kErrAttnWait);
      issue(kbase, S.kt[st], &S.kfull[st], t);
    }
  } else if (vprod) {
    // ---------------- V producer ----------------
    for (int t = kAttnStages; t < ntiles; ++t) {
      const int st = t % kAttnStages;
      mbar_wait(&S.vempty[st], uint32_t(t / kAttnStages - 1) & 1u, a.ctl, kErrAttnWait);
      issue(vbase, S.vt[st], &S.vfull[st], t);
    }
  }
  __syncwarp();  // producer warps: lane 0 rejoins its warp before the barrier
  __syncthreads();
  if (tid == 0) attn_time_end(a.ctl, timing);
}

// Sequence split, inside the combine: this rank's record (lanes 0-7 of warp
// w hold dims 8w..8w+7 of the CTA's 32 unnormalised o values; m, l) goes to
// every rank's receive buffer, then a flag tagged (epoch, pos + 1) per rank;
// the CTA waits (bounded) for every rank's flag and merges the records in
// rank order: M = max m_q, f_q = e^(m_q - M), o = sum f_q o_q / sum f_q l_q.
// Every rank merges the same records in the same order, so all ranks get
// the same bits. Returns the lane's normalised value.
constexpr unsigned long long kXWaitNs = 10ull * 1000 * 1000 * 1000;  // default bound: 10 s
__device__ __noinline__ float x_exchange(const AttnArgs& a, float r, float m, float l, uint32_t pos) {
  constexpr float kMin = -3.4028234663852886e38f;
  __shared__ int xfail;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.xworld, R = a.xrank;
  const int slot = a.xlayer * 2 + int(pos & 1u);
  const int cta = blockIdx.x * gridDim.y + blockIdx.y;
  const unsigned long long tag = (static_cast<unsigned long long>(ld_cg_u32(&a.ctl->epoch)) << 32) | (pos + 1u);
  for (int p = 0; p < G; ++p) {
    float* dst = a.xrecv[p] + x_rec_off(slot, R, cta, G);
    if (lane < 8) dst[warp * 8 + lane] = r;
    if (tid == 0) {
      dst[32] = m;
      dst[33] = l;
    }
  }
  if (tid == 0) xfail = 0;
  __syncthreads();
  if (tid < G) {
    __threadfence_system();
    st_release_sys_u64(a.xflag[tid] + x_flag_off(slot, R, cta, G), tag);
    const unsigned long long* f = a.xflag[R] + x_flag_off(slot, tid, cta, G);
    // after any expired wait of this session (err set) the rest of the
    // queued work falls through instead of waiting again
    const unsigned long long t0 = globaltimer_ns();
    const unsigned long long limit = a.xwait_ms ? a.xwait_ms * 1000000ull : kXWaitNs;
    while (ld_acquire_sys_u64(f) != tag) {
      if (ld_cg_u32(&a.ctl->err) != 0u) {
        xfail = 1;
        break;
      }
      if (globaltimer_ns() - t0 > limit) {
        atomicCAS(&a.ctl->err, 0u, kErrXWait);
        xfail = 1;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  if (xfail || lane >= 8) return 0.0f;
  const float* rec = a.xrecv[R] + x_rec_off(slot, 0, cta, G);
  const size_t src_stride = size_t(kXCtas) * kXRec;
  float M = kMin;
  for (int q = 0; q < G; ++q) M = fmaxf(M, __ldcv(rec + q * src_stride + 32));
  float L = 0.0f, O = 0.0f;
  for (int q = 0; q < G; ++q) {
    const float* rq = rec + q * src_stride;
    const float f = fexp(__fsub_rn(__ldcv(rq + 32), M));
    L = __fadd_rn(L, __fmul_rn(f, __ldcv(rq + 33)));
    O = __fadd_rn(O, __fmul_rn(f, __ldcv(rq + warp * 8 + lane)));
  }
  return L == 0.0f ? O : __fdiv_rn(O, L);
}

// Chain combine and BF16 output gate. Grid (8 query heads, 8 stripes of 32
// dims), 4 warps of 8 dims: the reference's attn_decode_split2_gate SIMD
// layout (lane l owns chains l and l+32, attention_decode.metal:853-889), or
// sdpa_vector's final reduction (lane l = chain l, :194-212) below 1024 keys,
// followed by attn_gate (attention.metal:140-150).
template <bool SESS>
__global__ void __launch_bounds__(128) k_attn_combine(const __grid_constant__ AttnArgs a_in) {
  AttnArgs sv;
  if constexpr (SESS) sv = attn_session_view(a_in, blockIdx.z);
  const AttnArgs& a = SESS ? sv : a_in;
  constexpr float kMin = -3.4028234663852886e38f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int qh = blockIdx.x, kh = qh >> 2, h = qh & 3;
  const int stripe = blockIdx.y * 4 + warp;  // 8 dims
  // Before the wait: the step's position (written by its first launch) and
  // the output gate (its input written by the q/k/v projection, two launches
  // back), so neither load sits after the dependency wait.
  const uint32_t len = ld_cg_u32(&a.ctl->pos_step) + uint32_t(a.pos_add) + 1;
  const float gate = lane < 8 ? attn_gate_bf(bf2f(a.q_raw[qh * 512 + 256 + stripe * 8 + lane])) : 0.0f;
  pdl_wait();
  pdl_launch();
  const bool xs = a.xworld > 1;
  const bool split = xs || len >= 1024;
  const size_t base = size_t(kh) * kAttnChains * 4 + h;  // + chain * 4
  float res[8];
  float xm = 0.0f, xl = 0.0f;  // sequence split: this rank's max and sum
  if (split) {
    const size_t ia = base + size_t(lane) * 4, ib = base + size_t(lane + 32) * 4;
    const float2 mla = *reinterpret_cast<const float2*>(&a.part_ml[ia * 2]);
    const float2 mlb = *reinterpret_cast<const float2*>(&a.part_ml[ib * 2]);
    const float4 pa0 = *reinterpret_cast<const float4*>(a.part_o + ia * kHeadDim + stripe * 8);
    const float4 pa1 = *reinterpret_cast<const float4*>(a.part_o + ia * kHeadDim + stripe * 8 + 4);
    const float4 pb0 = *reinterpret_cast<const float4*>(a.part_o + ib * kHeadDim + stripe * 8);
    const float4 pb1 = *reinterpret_cast<const float4*>(a.part_o + ib * kHeadDim + stripe * 8 + 4);
    const float pa[8] = {pa0.x, pa0.y, pa0.z, pa0.w, pa1.x, pa1.y, pa1.z, pa1.w};
    const float pb[8] = {pb0.x, pb0.y, pb0.z, pb0.w, pb1.x, pb1.y, pb1.z, pb1.w};
    const float M = warp_max(fmaxf(fmaxf(kMin, mla.x), mlb.x));
    const float fa = fexp(__fsub_rn(mla.x, M)), fb = fexp(__fsub_rn(mlb.x, M));
    float sacc = __fadd_rn(0.0f, __fmul_rn(fa, mla.y));
    sacc = __fadd_rn(sacc, __fmul_rn(fb, mlb.y));
    const float ssum_all = warp_sum(sacc);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float acc = __fadd_rn(0.0f, __fmul_rn(fa, pa[i]));
      acc = __fadd_rn(acc, __fmul_rn(fb, pb[i]));
      const float ov = warp_sum(acc);
      res[i] = (xs || ssum_all == 0.0f) ? ov : __fdiv_rn(ov, ssum_all);
    }
    xm = M;
    xl = ssum_all;
  } else {
    const size_t il = base + size_t(lane) * 4;
    const float2 ml = *reinterpret_cast<const float2*>(&a.part_ml[il * 2]);
    const float4 p0 = *reinterpret_cast<const float4*>(a.part_o + il * kHeadDim + stripe * 8);
    const float4 p1 = *reinterpret_cast<const float4*>(a.part_o + il * kHeadDim + stripe * 8 + 4);
    const float pl[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const float M = warp_max(ml.x);
    const float fl = fexp(__fsub_rn(ml.x, M));
    const float ssum_all = warp_sum(__fmul_rn(ml.y, fl));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float ov = warp_sum(__fmul_rn(pl[i], fl));
      res[i] = ssum_all == 0.0f ? ov : __fdiv_rn(ov, ssum_all);
    }
  }
  float r = res[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) r = lane == i ? res[i] : r;
  if (xs) r = x_exchange(a, r, xm, xl, len - 1);
  if (lane < 8) {
    const int d = stripe * 8 + lane;
    const float attention = bfr(r);
    a.gated[qh * kHeadDim + d] = f2bf(__fmul_rn(attention, gate));
  }
}

// Sets the control block of a standalone attention call: the position and
// its RoPE table (the decode step's first launch does this in-line).
__global__ void k_ctl_position(Ctl* ctl, uint32_t pos) {
  if (threadIdx.x == 0) {
    ctl->pos_step = pos;
    ctl->pos = pos;
    ctl->err = 0;
    ctl->attn_counter[0] = 0;
    ctl->attn_counter[1] = 0;
    ctl->head_counter = 0;
    ctl->out_count = 0;
    ctl->timing_on = 0;
  }
  if (threadIdx.x < 32) rope_pair(pos, threadIdx.x, ctl->rope_cs);
}

// ---------------------------------------------------------------------------
// Vocabulary head: final RMSNorm, Q4 projection of 248,320 tied-embedding
// rows streamed through a bulk-copy ring, per-CTA online (max, sum exp), then
// the last-arriving CTA forms lse = bf16(log(sum) + max) and picks the lowest
// id among the maxima of bf16(logit - lse) (head_lse.metal:66-98). Only CTAs
// whose own maximum reaches the winning value are rescanned.
// ---------------------------------------------------------------------------
// Last-CTA tail shared by the head and the standalone greedy kernel:
// lse = bf16(log(sum) + max) from the per-CTA (max, sum) partials, then the
// lowest id among the maxima of bf16(logit - lse) (head_lse.metal:66-98).
// Only the first CTA whose own maximum reaches the winning value is rescanned.
__device__ void head_finish(const HeadArgs& a, float* red, uint32_t* cand, uint32_t* best) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __threadfence();
  if (warp == 0) {
    float M = -INFINITY;
    for (int c = lane; c < int(gridDim.x); c += 32) M = fmaxf(M, __ldcg(&a.part[2 * c]));
    M = warp_max(M);
    float s = 0.0f;
    for (int c = lane; c < int(gridDim.x); c += 32) {
      const float sc = __ldcg(&a.part[2 * c + 1]);
      if (sc > 0.0f) s = __fmaf_rn(sc, expf(__ldcg(&a.part[2 * c]) - M), s);
    }
    s = warp_sum(s);
    if (lane == 0) {
      const uint16_t lse = f2bf(__fadd_rn(dlogf(s), M));
      red[0] = bf2f(lse);
      red[1] = bfr(__fsub_rn(M, bf2f(lse)));
      *cand = 0xffffffffu;
      *best = 0xffffffffu;
      if (a.lse_out) a.lse_out[0] = lse;
    }
  }
  __syncthreads();
  const float lse = red[0], W = red[1];
  for (int c = tid; c < int(gridDim.x); c += blockDim.x)
    if (bfr(__fsub_rn(__ldcg(&a.part[2 * c]), lse)) == W) atomicMin(cand, uint32_t(c));
  __syncthreads();
  const uint32_t c = *cand;
  if (c != 0xffffffffu) {
    const int rb = int(c) * kHeadRowsPerCta;
    const int re = min(kVocab, rb + kHeadRowsPerCta);
    for (int r = rb + tid; r < re; r += blockDim.x) {
      const float lv = bf2f(__ldcg(&a.logits[r]));
      if (bfr(__fsub_rn(lv, lse)) == W) atomicMin(best, uint32_t(r));
    }
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t token = *best == 0xffffffffu ? 0u : *best;
    Ctl* ctl = a.ctl;
    const uint32_t ps = ctl->pos_step;
    if (a.seq && ps + 1 < a.seq_len) a.seq[ps + 1] = token;
    const uint32_t oc = ctl->out_count;
    if (a.out_tokens && oc < a.out_len) a.out_tokens[oc] = token;
    ctl->out_count = oc + 1;
    ctl->head_counter = 0;
  }
}

// Online (max, sum exp) of one thread's logits, one logit at a time.
__device__ __forceinline__ void lse_push(float& run_m, float& run_s, float lv) {
  if (lv > run_m) {
    run_s = __fmaf_rn(run_s, __expf(run_m - lv), 1.0f);
    run_m = lv;
  } else {
    run_s += __expf(lv - run_m);
  }
}

// Warp-level (max, sum exp) of the lanes' online states (warp butterfly).
__device__ __forceinline__ void lse_warp(float run_m, float run_s, float& M, float& S) {
  M = warp_max(run_m);
  const float s = run_s > 0.0f ? run_s * __expf(run_m - M) : 0.0f;
  S = warp_sum(s);
}

// One thread: the CTA's (max, sum exp) from its warps' partials, stored as
// the CTA's grid partial; returns whether this CTA arrived last.
__device__ __forceinline__ bool lse_cta(const float* wm, const float* ws, int nw, float* part,
                                        uint32_t* counter) {
  float MM = wm[0];
  for (int w = 1; w < nw; ++w) MM = fmaxf(MM, wm[w]);
  float ss = 0.0f;
  for (int w = 0; w < nw; ++w)
    if (ws[w] > 0.0f) ss = __fmaf_rn(ws[w], __expf(wm[w] - MM), ss);
  part[2 * blockIdx.x] = MM;
  part[2 * blockIdx.x + 1] = ss;
  __threadfence();
  return atomicAdd(counter, 1u) == gridDim.x - 1;
}

// Per-CTA (max, sum exp) of a row range of bf16 logits, combined into the
// CTA's partial; returns whether this CTA arrived last.
__device__ bool head_partial(const HeadArgs& a, float run_m, float run_s, float* wm, float* ws,
                             int* last) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float M, S;
  lse_warp(run_m, run_s, M, S);
  if (lane == 0) {
    wm[warp] = M;
    ws[warp] = S;
  }
  __syncthreads();
  if (tid == 0) *last = lse_cta(wm, ws, blockDim.x / 32, a.part, &a.ctl->head_counter);
  __syncthreads();
  return *last != 0;
}

struct HeadSmem {
  uint32_t codes[kHeadStages][kHeadRowsPerChunk * 128];
  uint16_t scl[kHeadStages][kHeadRowsPerChunk * 16];
  uint16_t bia[kHeadStages][kHeadRowsPerChunk * 16];
  float4 xq[2 * 4 * 32];
  float xsum[2 * 32];
  float xf[kHidden];
  float red[64];
  float wm[kHeadThreads / 32], ws[kHeadThreads / 32];
  uint64_t bar[kHeadStages];
  uint32_t done[kHeadStages];  // warps finished with each ring stage
  int last;
  uint32_t cand;
  uint32_t best;
};
size_t head_smem_bytes() { return sizeof(HeadSmem); }

__global__ void __launch_bounds__(kHeadThreads, 1) k_head(const __grid_constant__ HeadArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  HeadSmem& S = *reinterpret_cast<HeadSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kHeadRowsPerCta;
  const int nrows = min(kHeadRowsPerCta, kVocab - r0);
  const int nchunks = (nrows + kHeadRowsPerChunk - 1) / kHeadRowsPerChunk;
  auto issue = [&](int ch, int st) {
    const int rows = min(kHeadRowsPerChunk, nrows - ch * kHeadRowsPerChunk);
    const size_t row = size_t(r0) + size_t(ch) * kHeadRowsPerChunk;
    mbar_expect_tx(&S.bar[st], uint32_t(rows) * (512 + 64));
    bulk_g2s(S.codes[st], a.w + row * 128, uint32_t(rows) * 512, &S.bar[st]);
    bulk_g2s(S.scl[st], a.s + row * 16, uint32_t(rows) * 32, &S.bar[st]);
    bulk_g2s(S.bia[st], a.b + row * 16, uint32_t(rows) * 32, &S.bar[st]);
  };
  if (tid == 0) {
    for (int s = 0; s < kHeadStages; ++s) {
      mbar_init(&S.bar[s], 1);
      S.done[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int s = 0; s < kHeadStages && s < nchunks; ++s) issue(s, s);
  const bool holder = tid < kHidden / 4;  // threads 0-255 hold four activations each
  float g[4] = {1.f, 1.f, 1.f, 1.f};
  if (a.gain && holder) {
    const float4 g4 = bf4(*reinterpret_cast<const uint2*>(a.gain + 4 * tid));
    g[0] = g4.x, g[1] = g4.y, g[2] = g4.z, g[3] = g4.w;
  }
  pdl_wait();
  pdl_launch();
  {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (holder) {
      const float4 x4 = bf4(*reinterpret_cast<const uint2*>(a.x + 4 * tid));
      v[0] = x4.x, v[1] = x4.y, v[2] = x4.z, v[3] = x4.w;
    }
    if (a.gain) {
      float o[4];
      rms1024_reg(v, g, o, S.red);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = o[j];
    }
    if (holder) *reinterpret_cast<float4*>(S.xf + 4 * tid) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  build_xq(S.xf, kHidden, S.xq, S.xsum);
  __syncthreads();
  // the lane's constants of both 512-wide halves stay in registers
  float4 xx0[4], cc0[4], xx1[4], cc1[4];
  float xs0, xs1;
  load_xq(S.xq, S.xsum, 0, lane, xx0, cc0, xs0);
  load_xq(S.xq, S.xsum, 1, lane, xx1, cc1, xs1);

  // Warp w owns rows 4w..4w+3 of every chunk: both 512-wide halves,
  // the cross-lane finish and the logits, with no block barrier. The last
  // warp done with a ring stage refills it. Lanes 0-3 keep the online
  // (max, sum exp) of their row.
  float run_m = -INFINITY, run_s = 0.0f;
  const int g0 = 4 * warp;
  for (int ch = 0; ch < nchunks; ++ch) {
    const int st = ch % kHeadStages;
    mbar_wait(&S.bar[st], uint32_t(ch / kHeadStages) & 1u, a.ctl, kErrHeadWait);
    const int rows = min(kHeadRowsPerChunk, nrows - ch * kHeadRowsPerChunk);
    float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
    if (g0 < rows) {
      qmv_rows_terms(S.codes[st], S.scl[st], S.bia[st], rows, g0, 0, kHidden, xx0, cc0, xs0, lane, t0);
      qmv_rows_terms(S.codes[st], S.scl[st], S.bia[st], rows, g0, 1, kHidden, xx1, cc1, xs1, lane, t1);
    }
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&S.done[st], 1u) == uint32_t(kHeadThreads / 32 - 1)) {
        S.done[st] = 0;
        if (ch + kHeadStages < nchunks) {
          fence_proxy_async();
          issue(ch + kHeadStages, st);
        }
      }
    }
    if (g0 < rows) {
      // the lane's two chunk terms summed from 0 in chunk order (the finish of
      // qmv_finish_task, kept in registers), then the rows' butterflies:
      // row j ends on lane 16 (j >> 1) + 8 (j & 1)
      const float v = reduce4(__fadd_rn(__fadd_rn(0.0f, t0[0]), t1[0]), __fadd_rn(__fadd_rn(0.0f, t0[1]), t1[1]),
                              __fadd_rn(__fadd_rn(0.0f, t0[2]), t1[2]), __fadd_rn(__fadd_rn(0.0f, t0[3]), t1[3]),
                              lane);
      const float vr = __shfl_sync(0xffffffffu, v, ((lane & 2) << 3) | ((lane & 1) << 3));
      if (lane < 4 && g0 + lane < rows) {
        const uint16_t lb = f2bf(vr);
        a.logits[r0 + ch * kHeadRowsPerChunk + g0 + lane] = lb;
        lse_push(run_m, run_s, bf2f(lb));
      }
    }
    __syncwarp();
  }
  head_partial(a, run_m, run_s, S.wm, S.ws, &S.last);
  if (!S.last) return;
  head_finish(a, S.red, &S.cand, &S.best);
}


// Vocabulary head for up to kMaxSessions sessions at once: the head's chunk
// ring streams each weight row once and applies it to every session; per
// session the logits, the online (max, sum exp) of lanes 4t..4t+3 (rows
// 0..3 of a warp's four, as lanes 0..3 in k_head), the CTA and grid
// combines and the greedy tail are those of k_head, so each session's
// result equals a single-session head's bit for bit.
constexpr int kHeadBStages = 3;
struct HeadBatchSmem {
  uint32_t codes[kHeadBStages][kHeadRowsPerChunk * 128];
  uint16_t scl[kHeadBStages][kHeadRowsPerChunk * 16];
  uint16_t bia[kHeadBStages][kHeadRowsPerChunk * 16];
  float xf[kMaxSessions][kHidden];
  float4 xq[kMaxSessions][2 * 4 * 32];
  float xsum[kMaxSessions][2 * 32];
  float red[64];
  float wm[kMaxSessions][kHeadThreads / 32], ws[kMaxSessions][kHeadThreads / 32];
  uint64_t bar[kHeadBStages];
  uint32_t done[kHeadBStages];
  int last[kMaxSessions];
  uint32_t cand;
  uint32_t best;
};
size_t head_batch_smem_bytes() { return sizeof(HeadBatchSmem); }

__global__ void __launch_bounds__(kHeadThreads, 1) k_head_batch(const __grid_constant__ HeadBatchArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  HeadBatchSmem& S = *reinterpret_cast<HeadBatchSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = a.n;
  const int r0 = blockIdx.x * kHeadRowsPerCta;
  const int nrows = min(kHeadRowsPerCta, kVocab - r0);
  const int nchunks = (nrows + kHeadRowsPerChunk - 1) / kHeadRowsPerChunk;
  auto issue = [&](int ch, int st) {
    const int rows = min(kHeadRowsPerChunk, nrows - ch * kHeadRowsPerChunk);
    const size_t row = size_t(r0) + size_t(ch) * kHeadRowsPerChunk;
    mbar_expect_tx(&S.bar[st], uint32_t(rows) * (512 + 64));
    bulk_g2s(S.codes[st], a.w + row * 128, uint32_t(rows) * 512, &S.bar[st]);
    bulk_g2s(S.scl[st], a.s + row * 16, uint32_t(rows) * 32, &S.bar[st]);
    bulk_g2s(S.bia[st], a.b + row * 16, uint32_t(rows) * 32, &S.bar[st]);
  };
  if (tid == 0) {
    for (int s = 0; s < kHeadBStages; ++s) {
      mbar_init(&S.bar[s], 1);
      S.done[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int s = 0; s < kHeadBStages && s < nchunks; ++s) issue(s, s);
  pdl_wait();
  pdl_launch();
  // final RMSNorm of session `warp` (the warp-level form of rms1024_reg)
  if (warp < n) {
    float gain[8][4];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const float4 g4 = a.gain ? bf4(*reinterpret_cast<const uint2*>(a.gain + 128 * s + 4 * lane))
                               : make_float4(1.f, 1.f, 1.f, 1.f);
      gain[s][0] = g4.x, gain[s][1] = g4.y, gain[s][2] = g4.z, gain[s][3] = g4.w;
    }
    float v[8][4];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const float4 x4 = bf4(*reinterpret_cast<const uint2*>(a.x + size_t(warp) * kHidden + 128 * s + 4 * lane));
      v[s][0] = x4.x, v[s][1] = x4.y, v[s][2] = x4.z, v[s][3] = x4.w;
    }
    const float inv = a.gain ? rms1024_warp_inv(v) : 1.0f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = a.gain ? bfr(__fmul_rn(bfr(__fmul_rn(v[s][j], inv)), gain[s][j])) : v[s][j];
      *reinterpret_cast<float4*>(&S.xf[warp][128 * s + 4 * lane]) = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();
  for (int t = 0; t < n; ++t) build_xq(S.xf[t], kHidden, S.xq[t], S.xsum[t]);
  __syncthreads();

  float run_m = -INFINITY, run_s = 0.0f;  // lane 4t + r: session t, row r of the warp's four
  const int g0 = 4 * warp, my_t = lane >> 2, my_r = lane & 3;
  for (int ch = 0; ch < nchunks; ++ch) {
    const int st = ch % kHeadBStages;
    mbar_wait(&S.bar[st], uint32_t(ch / kHeadBStages) & 1u, a.out[0].ctl, kErrHeadWait);
    const int rows = min(kHeadRowsPerChunk, nrows - ch * kHeadRowsPerChunk);
    float mine = 0.0f;
    if (g0 < rows) {
      // sessions in blocks of kBlockTokens: each block decodes the rows once
#pragma unroll 1
      for (int j0 = 0; j0 < n; j0 += kBlockTokens) {
        const int nj = min(kBlockTokens, n - j0);
        float acc[kBlockTokens][4];
#pragma unroll
        for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[j][r] = 0.0f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float term[kBlockTokens][4];
          qmv_block_terms(S.codes[st], S.scl[st], S.bia[st], rows, g0, c, kHidden / 8, kHidden / 64, 2,
                          &S.xq[0][0], &S.xsum[0][0], j0, nj, lane, term);
#pragma unroll
          for (int j = 0; j < kBlockTokens; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[j][r] = __fadd_rn(acc[j][r], term[j][r]);
        }
#pragma unroll
        for (int j = 0; j < kBlockTokens; ++j) {
          if (j < nj) {
            const float v = reduce4(acc[j][0], acc[j][1], acc[j][2], acc[j][3], lane);  // row r in lane 8r
            const float vr = __shfl_sync(0xffffffffu, v, 8 * my_r);
            if (my_t == j0 + j) mine = vr;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&S.done[st], 1u) == uint32_t(kHeadThreads / 32 - 1)) {
        S.done[st] = 0;
        if (ch + kHeadBStages < nchunks) {
          fence_proxy_async();
          issue(ch + kHeadBStages, st);
        }
      }
    }
    if (my_t < n && g0 + my_r < rows) {
      const uint16_t lb = f2bf(mine);
      a.out[my_t].logits[r0 + ch * kHeadRowsPerChunk + g0 + my_r] = lb;
      lse_push(run_m, run_s, bf2f(lb));
    }
    __syncwarp();
  }
  // per session: warp and CTA combines, then the grid tail on its last CTA
  for (int t = 0; t < n; ++t) {
    float M, Ssum;
    lse_warp(my_t == t ? run_m : -INFINITY, my_t == t ? run_s : 0.0f, M, Ssum);
    if (lane == 0) {
      S.wm[t][warp] = M;
      S.ws[t][warp] = Ssum;
    }
  }
  __syncthreads();
  if (tid < n) S.last[tid] = lse_cta(S.wm[tid], S.ws[tid], kHeadThreads / 32, a.out[tid].part,
                                     &a.out[tid].ctl->head_counter);
  __syncthreads();
  for (int t = 0; t < n; ++t) {
    if (!S.last[t]) continue;
    HeadArgs v = {};
    v.logits = a.out[t].logits;
    v.part = a.out[t].part;
    v.seq = a.out[t].seq;
    v.out_tokens = a.out[t].out_tokens;
    v.seq_len = a.out[t].seq_len;
    v.out_len = a.out[t].out_len;
    v.lse_out = a.out[t].lse;
    v.ctl = a.out[t].ctl;
    head_finish(v, S.red, &S.cand, &S.best);
  }
}

// Greedy selection on given logits (greedy_bf16, linear.metal:400-449), with
// the head's partition and tail.
__global__ void __launch_bounds__(256) k_greedy(const __grid_constant__ HeadArgs a) {
  __shared__ float red[64], wm[8], ws[8];
  __shared__ int last;
  __shared__ uint32_t cand, best;
  const int r0 = blockIdx.x * kHeadRowsPerCta;
  const int r1 = min(kVocab, r0 + kHeadRowsPerCta);
  float run_m = -INFINITY, run_s = 0.0f;
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    lse_push(run_m, run_s, bf2f(a.logits[r]));
  }
  if (!head_partial(a, run_m, run_s, wm, ws, &last)) return;
  head_finish(a, red, &cand, &best);
}

// Greedy selection for batched sessions: grid (148, n), session blockIdx.y
// runs k_greedy's partition and tail on its own logits row and outputs.
__global__ void __launch_bounds__(256) k_greedy_sessions(const HeadOut* __restrict__ outs) {
  __shared__ float red[64], wm[8], ws[8];
  __shared__ int last;
  __shared__ uint32_t cand, best;
  const HeadOut& o = outs[blockIdx.y];
  HeadArgs a = {};
  a.logits = o.logits;
  a.part = o.part;
  a.seq = o.seq;
  a.out_tokens = o.out_tokens;
  a.seq_len = o.seq_len;
  a.out_len = o.out_len;
  a.lse_out = o.lse;
  a.ctl = o.ctl;
  pdl_wait();
  pdl_launch();
  const int r0 = blockIdx.x * kHeadRowsPerCta;
  const int r1 = min(kVocab, r0 + kHeadRowsPerCta);
  float run_m = -INFINITY, run_s = 0.0f;
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) lse_push(run_m, run_s, bf2f(a.logits[r]));
  if (!head_partial(a, run_m, run_s, wm, ws, &last)) return;
  head_finish(a, red, &cand, &best);
}

cudaError_t launch_greedy_sessions(const HeadOut* outs, int n, cudaStream_t st, bool pdl) {
  return launch_ex(k_greedy_sessions, dim3(kHeadCtas, n), dim3(256), 0, st, pdl, outs);
}

// Diagnostic: the bounded mbarrier wait every kernel uses, on a barrier that
// nothing ever completes, with a caller-chosen poll limit. The wait gives up,
// records kErrProbeWait in *err and the kernel returns normally (no copy is
// in flight, so leaving the barrier pending is harmless).
__global__ void k_wait_probe(uint32_t polls, uint32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait_limit(&bar, 0, polls, err, kErrProbeWait);
}

// Embedding row (linear.metal:11-24), standalone op.
__global__ void k_embedding(const uint32_t* w, const uint16_t* s, const uint16_t* b, uint32_t token,
                            int K, uint16_t* out) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  const uint32_t q = (w[size_t(token) * (K / 8) + k / 8] >> (4 * (k % 8))) & 15u;
  const size_t g = size_t(token) * (K / 64) + k / 64;
  out[k] = f2bf(__fadd_rn(__fmul_rn(bf2f(s[g]), float(q)), bf2f(b[g])));
}

// RMSNorm of one 1024 vector, standalone op (same device path as the fused
// prologues).
__global__ void __launch_bounds__(256) k_rms1024(const uint16_t* x, const uint16_t* gain,
                                                 uint16_t* out) {
  __shared__ float xf[kHidden];
  __shared__ float red[64];
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = bf2f(x[4 * threadIdx.x + j]);
  rms1024(v, gain, xf, red);
#pragma unroll
  for (int j = 0; j < 4; ++j) out[4 * threadIdx.x + j] = f2bf(xf[4 * threadIdx.x + j]);
}

// ---------------------------------------------------------------------------
// host-side launch helpers
// ---------------------------------------------------------------------------

// Dynamic shared memory requested by every kernel of the decode step: more
// than half an SM's 228 KB, so one CTA fits per SM and every kernel's
// 128-148 CTAs land on distinct SMs. With room for two or more, the block
// scheduler packed a kernel launched early (programmatic launch) three or
// four CTAs to an SM onto the SMs its predecessor left free (measured: 144
// CTAs on 39 SMs), multiplying that kernel's time; one CTA per SM costs only
// the overlap of a CTA's weight prefetch with the predecessor on that SM.
constexpr size_t kSpreadSmem = 115 * 1024;
static size_t spread(size_t bytes) { return bytes < kSpreadSmem ? kSpreadSmem : bytes; }

// The (prologue, epilogue) pairs the decode step and the op entry points use.
#define Q35_QMV_VARIANTS(X)         \
  X(kProEmbedRms, kEpiGdnConv)      \
  X(kProRms, kEpiGdnConv)           \
  X(kProRms, kEpiStore)             \
  X(kProRms, kEpiSwiglu)            \
  X(kProNormGate, kEpiResAdd)       \
  X(kProNormGate, kEpiStore)        \
  X(kProPlain, kEpiResAdd)          \
  X(kProPlain, kEpiStore)
static void (*qmv_kernel(int pro, int epi))(QmvArgs) {
#define Q35_QMV_PICK(P, E) \
  if (pro == P && epi == E) return k_qmv<P, E>;
  Q35_QMV_VARIANTS(Q35_QMV_PICK)
#undef Q35_QMV_PICK
  return nullptr;
}
template <class F>
static cudaError_t for_each_qmv(F f) {
  cudaError_t e = cudaSuccess;
#define Q35_QMV_EACH(P, E) \
  if (e == cudaSuccess) e = f(k_qmv<P, E>);
  Q35_QMV_VARIANTS(Q35_QMV_EACH)
#undef Q35_QMV_EACH
  return e;
}

cudaError_t kernels_init() {
  cudaError_t e;
  e = for_each_qmv([](auto kern) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSpreadSmem));
  });
  if (e != cudaSuccess) return e;
  for (auto kern : {k_attn<false>, k_attn<true>}) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(spread(attn_smem_bytes())));
    if (e != cudaSuccess) return e;
  }
  e = cudaFuncSetAttribute(k_head, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(spread(head_smem_bytes())));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_head_batch, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(spread(head_batch_smem_bytes())));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_gdn_recur, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(kSpreadSmem));
  if (e != cudaSuccess) return e;
  for (auto kern : {k_attn_combine<false>, k_attn_combine<true>}) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSpreadSmem));
    if (e != cudaSuccess) return e;
  }
  return e;
}

int qmv_max_rows(int K) {
  int r = 1;  // the epilogue gives each CTA row its own thread
  while (r < kQmvThreads && qmv_layout(K, r + 1).total <= kSpreadSmem) ++r;
  return r;
}

cudaError_t launch_qmv(const QmvArgs& a, cudaStream_t st, bool pdl) {
  const int grid = (a.units + a.units_per_cta - 1) / a.units_per_cta;
  void (*kern)(QmvArgs) = qmv_kernel(a.pro, a.epi);
  if (!kern) return cudaErrorInvalidValue;
  return launch_ex(kern, dim3(grid), dim3(kQmvThreads), spread(qmv_smem_bytes(a)), st, pdl, a);
}
cudaError_t launch_recur(const RecurArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_gdn_recur, dim3(8, kGdnHeads), dim3(128), kSpreadSmem, st, pdl, a);
}
cudaError_t launch_attn(const AttnArgs& a_in, cudaStream_t st, bool pdl) {
  AttnArgs a = a_in;
  a.nzero = -0.0f;
  cudaError_t e = launch_ex(k_attn<false>, dim3(kAttnChains, kKvHeads), dim3(kAttnThreads),
                            spread(attn_smem_bytes()), st, pdl, a);
  if (e != cudaSuccess) return e;
  return launch_ex(k_attn_combine<false>, dim3(kQHeads, kHeadDim / 32), dim3(128), kSpreadSmem, st, true, a);
}
cudaError_t launch_attn_sessions(const AttnArgs& a_in, int n, cudaStream_t st, bool pdl) {
  AttnArgs a = a_in;
  a.nzero = -0.0f;
  if (n < 1 || !a.sess || a.xworld > 1 || !a.rope) return cudaErrorInvalidValue;
  cudaError_t e = launch_ex(k_attn<true>, dim3(kAttnChains, kKvHeads, n), dim3(kAttnThreads),
                            spread(attn_smem_bytes()), st, pdl, a);
  if (e != cudaSuccess) return e;
  return launch_ex(k_attn_combine<true>, dim3(kQHeads, kHeadDim / 32, n), dim3(128), kSpreadSmem, st, true, a);
}
cudaError_t launch_head(const HeadArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_head, dim3(kHeadCtas), dim3(kHeadThreads), spread(head_smem_bytes()), st, pdl, a);
}
cudaError_t launch_head_batch(const HeadBatchArgs& a, cudaStream_t st, bool pdl) {
  if (a.n < 1 || a.n > kMaxSessions) return cudaErrorInvalidValue;
  return launch_ex(k_head_batch, dim3(kHeadCtas), dim3(kHeadThreads), spread(head_batch_smem_bytes()), st,
                   pdl, a);
}
cudaError_t launch_greedy(const HeadArgs& a, cudaStream_t st) {
  return launch_ex(k_greedy, dim3(kHeadCtas), dim3(256), 0, st, false, a);
}
cudaError_t launch_gdn_conv(const uint16_t* raw, uint16_t* hist, const uint16_t* convw,
                            uint16_t* conv_out, cudaStream_t st) {
  k_gdn_conv<<<kGdnConv / 256, 256, 0, st>>>(raw, hist, convw, conv_out);
  return cudaGetLastError();
}
cudaError_t launch_wait_probe(uint32_t polls, uint32_t* err, cudaStream_t st) {
  k_wait_probe<<<1, 32, 0, st>>>(polls, err);
  return cudaGetLastError();
}
cudaError_t launch_ctl_position(Ctl* ctl, uint32_t pos, cudaStream_t st) {
  k_ctl_position<<<1, 32, 0, st>>>(ctl, pos);
  return cudaGetLastError();
}
cudaError_t launch_embedding(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                             uint32_t token, int K, uint16_t* out, cudaStream_t st) {
  k_embedding<<<(K + 255) / 256, 256, 0, st>>>(w, s, b, token, K, out);
  return cudaGetLastError();
}
cudaError_t launch_rms1024(const uint16_t* x, const uint16_t* gain, uint16_t* out,
                           cudaStream_t st) {
  k_rms1024<<<1, 256, 0, st>>>(x, gain, out);
  return cudaGetLastError();
}

}  // namespace q35
