// Prompt chunks on the tensor cores: T consecutive prompt tokens of one
// session per chunk (the reference's prefill, model.rs:100-110 with 2048-row
// chunks, :189-198 GEMM route, :233-289 layer body). The projections are the
// tcgen05 GEMMs of q35_gemm.cu over the chunk and the per-token norms and
// activations those of q35_tokens.cu; this file holds the steps that walk the
// chunk:
//   k_pr_conv        GDN causal conv + SiLU of every token (gdn.metal:33-52),
//                    tokens in parallel (each output reads four raw rows)
//   k_pr_gdn_prep    q/k L2 scaling, decay gate and beta (gdn.metal:75-114),
//                    the z gate, and the conv history shift (gdn.metal:56-71)
//   k_pr_recur       the delta-rule recurrence over the chunk's tokens in
//                    order (gdn.metal:176-228), state in registers, inputs
//                    staged through a bulk-copy ring
//   k_pr_attn_prep   per-head q/k RMSNorm + partial RoPE, K/V appended to the
//                    cache (attention.metal:72-131)
//   k_pr_attn        causal flash attention on the tensor cores
//                    (attention_prefill.metal:1830-2258): 128 query rows
//                    (4 heads sharing a KV head x 32 tokens) against 64-key
//                    tiles, S = Q K^T and O += P V by tcgen05.mma with S and O
//                    in TMEM; two launches over each split's keys (row maxima;
//                    then P = exp(S - M) rounded to bf16 against the maximum
//                    M over all splits, and O), so O is never rescaled and
//                    every weight is the restatement's
//   k_pr_attn_combine  merges the key splits and applies the output gate
//                    (attention.metal:140-150)
// Every per-token step uses the decode step's device functions; only the
// GEMMs and the attention sum in the tensor core's order (and the attention
// weights are bf16), as the reference's own prefill does.
#include <cuda_runtime.h>

#include "q35_gdn.cuh"
#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_tc.cuh"
#include "q35_types.h"

namespace q35 {

// ---------------------------------------------------------------------------
// GDN layer
// ---------------------------------------------------------------------------

// grid (6144 / 512, ceil(T / 16)): thread = channel pair (2c, 2c + 1) for 16
// consecutive tokens; the 19 raw rows it needs (the three before the block
// from the history at the chunk's start) are loaded first as 32-bit pairs.
constexpr int kPrConvTokens = 16;
__global__ void __launch_bounds__(256) k_pr_conv(const __grid_constant__ PromptArgs a) {
  pdl_wait();
  pdl_launch();
  constexpr int P = kGdnConv / 2;  // channel pairs per row
  const int c = blockIdx.x * 256 + threadIdx.x;
  const int t0 = blockIdx.y * kPrConvTokens, t1 = min(a.T, t0 + kPrConvTokens);
  const uint32_t* raw = reinterpret_cast<const uint32_t*>(a.raw);
  const uint32_t* hist = reinterpret_cast<const uint32_t*>(a.hist);
  uint32_t r[kPrConvTokens + 3];
#pragma unroll
  for (int i = 0; i < kPrConvTokens + 3; ++i) {
    const int t = t0 - 3 + i;
    r[i] = t < 0 ? hist[(3 + t) * P + c] : t < t1 ? raw[size_t(t) * P + c] : 0u;
  }
  const uint16_t wa[4] = {a.convw[8 * c], a.convw[8 * c + 1], a.convw[8 * c + 2], a.convw[8 * c + 3]};
  const uint16_t wb[4] = {a.convw[8 * c + 4], a.convw[8 * c + 5], a.convw[8 * c + 6], a.convw[8 * c + 7]};
  uint32_t* conv = reinterpret_cast<uint32_t*>(a.conv);
#pragma unroll
  for (int i = 0; i < kPrConvTokens; ++i) {
    if (t0 + i >= t1) break;
    const uint16_t lo = gdn_conv_value(uint16_t(r[i]), uint16_t(r[i + 1]), uint16_t(r[i + 2]), uint16_t(r[i + 3]), wa);
    const uint16_t hi = gdn_conv_value(uint16_t(r[i] >> 16), uint16_t(r[i + 1] >> 16), uint16_t(r[i + 2] >> 16),
                                       uint16_t(r[i + 3] >> 16), wb);
    conv[size_t(t0 + i) * P + c] = uint32_t(lo) | (uint32_t(hi) << 16);
  }
}

// grid T, 16 warps: warp h prepares head h of token t (k and q normalised to
// kq[h][t], gate and beta to gb[h][t], the head's values to vv), the block its
// token's z gate; blocks also shift the conv history to the chunk's last three
// raw rows (k_pr_conv, which read it, has finished).
__global__ void __launch_bounds__(512) k_pr_gdn_prep(const __grid_constant__ PromptArgs a) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, h = tid >> 5;
  const uint16_t* conv = a.conv + size_t(t) * kGdnConv;
  float* kq = a.kq + (size_t(h) * a.tmax + t) * 256;
  gdn_qk_norm(conv, h, false, lane, kq);
  gdn_qk_norm(conv, h, true, lane, kq + 128);
  if (lane == 0) {
    const float g = gdn_gate(a.ab[t * 32 + h], a.dt_bias[h], dexpf(a.a_log[h]));
    const float b = gdn_beta(a.ab[t * 32 + 16 + h]);
    *reinterpret_cast<float2*>(a.gb + (size_t(h) * a.tmax + t) * 2) = make_float2(g, b);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int vrow = 4 * lane + i;
    a.vv[((size_t(h) * 8 + (vrow >> 4)) * a.tmax + t) * 16 + (vrow & 15)] =
        bf2f(conv[4096 + h * 128 + vrow]);
  }
  for (int i = tid; i < 2048; i += 512) a.zs[size_t(t) * 2048 + i] = gdn_zgate(bf2f(a.z[size_t(t) * 2048 + i]));
  for (int c = blockIdx.x * 512 + tid; c < kGdnConv; c += gridDim.x * 512) {
    uint16_t n[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int tt = a.T - 3 + j;
      n[j] = tt >= 0 ? a.raw[size_t(tt) * kGdnConv + c] : a.hist[(3 + tt) * kGdnConv + c];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) a.hist[j * kGdnConv + c] = n[j];
  }
}

// Recurrence: grid (8 row blocks, 16 heads) x 128 threads, 8 lanes per value
// row with 16 state values each (gdn_decay_dot8 / gdn_update_dot8: the decode
// step's sums in its order, half the work per lane), walking the chunk's tokens in
// order. Thread 0 streams blocks of kPromptRecSub tokens' k|q rows, gates and
// values through a ring of kPrRecStages stages.
constexpr int kPrRecStages = 3;
struct PrRecStage {
  float kq[kPromptRecSub][256];
  float gb[kPromptRecSub][2];
  float vv[kPromptRecSub][16];
};
constexpr size_t kPrRecSmem = sizeof(PrRecStage) * kPrRecStages;

__global__ void __launch_bounds__(128) k_pr_recur(const __grid_constant__ PromptArgs a) {
  extern __shared__ __align__(128) uint8_t dsm[];
  PrRecStage* stg = reinterpret_cast<PrRecStage*>(dsm);
  __shared__ __align__(8) uint64_t full[kPrRecStages];
  const int tid = threadIdx.x, rb = blockIdx.x, h = blockIdx.y;
  const int T = a.T, nsub = (T + kPromptRecSub - 1) / kPromptRecSub;
  const int row = tid >> 3, r = tid & 7, vrow = rb * 16 + row;
  if (tid == 0) {
    for (int s = 0; s < kPrRecStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch();
  auto issue = [&](int b) {
    PrRecStage& S = stg[b % kPrRecStages];
    uint64_t* bar = &full[b % kPrRecStages];
    const size_t t0 = size_t(b) * kPromptRecSub;
    mbar_expect_tx(bar, uint32_t(sizeof(PrRecStage)));
    bulk_g2s(S.kq, a.kq + (size_t(h) * a.tmax + t0) * 256, kPromptRecSub * 256 * 4, bar);
    bulk_g2s(S.gb, a.gb + (size_t(h) * a.tmax + t0) * 2, kPromptRecSub * 2 * 4, bar);
    bulk_g2s(S.vv, a.vv + ((size_t(h) * 8 + rb) * a.tmax + t0) * 16, kPromptRecSub * 16 * 4, bar);
  };
  if (tid == 0)
    for (int b = 0; b < kPrRecStages && b < nsub; ++b) issue(b);
  float* gstate = a.state + (size_t(h) * 128 + vrow) * 128 + r * 16;
  float s[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = reinterpret_cast<const float4*>(gstate)[i];
    s[4 * i] = v.x;
    s[4 * i + 1] = v.y;
    s[4 * i + 2] = v.z;
    s[4 * i + 3] = v.w;
  }
  bool ok = true;
  for (int b = 0; b < nsub; ++b) {
    const bool got =
        mbar_wait(&full[b % kPrRecStages], uint32_t(b / kPrRecStages) & 1u, a.ctl, kErrPromptWait);
    if (__syncthreads_or(!got)) {
      ok = false;
      break;
    }
    const PrRecStage& S = stg[b % kPrRecStages];
    const int n = min(kPromptRecSub, T - b * kPromptRecSub);
    uint16_t* y = a.y + size_t(b) * kPromptRecSub * 2048 + h * 128 + vrow;
    for (int i = 0; i < n; ++i) {
      const float memory = gdn_reduce8(gdn_decay_dot8(s, &S.kq[i][r * 16], S.gb[i][0]));
      const float delta = __fmul_rn(__fsub_rn(S.vv[i][row], memory), S.gb[i][1]);
      const float out = gdn_reduce8(gdn_update_dot8(s, &S.kq[i][r * 16], &S.kq[i][128 + r * 16], delta));
      if (r == 0) y[size_t(i) * 2048] = f2bf(out);
    }
    __syncthreads();  // stage b is free again
    if (tid == 0 && b + kPrRecStages < nsub) issue(b + kPrRecStages);
  }
  if (!ok) return;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    reinterpret_cast<float4*>(gstate)[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
}

// ---------------------------------------------------------------------------
// Attention layer
// ---------------------------------------------------------------------------

// grid T, 10 warps: warps 0-7 normalise and rotate query head w of token t
// into qn[w][t] (bf16: the decode step's values are bf16 already), warps 8-9
// key head w - 8 into the cache at position p0 + t, with its value row.
__global__ void __launch_bounds__(320) k_pr_attn_prep(const __grid_constant__ PromptArgs a) {
  __shared__ __align__(16) float nrm[10][256];
  __shared__ __align__(16) float out[10][256];
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* rope = a.rope + 64 * t;
  uint4 packed;
  if (warp < 8) {
    head_norm_rope(a.q_raw + size_t(t) * kQProj + warp * 512, a.q_gain, rope, nrm[warp], out[warp], lane);
  } else {
    head_norm_rope(a.k_raw + size_t(t) * 512 + (warp - 8) * 256, a.k_gain, rope, nrm[warp], out[warp], lane);
  }
  const float* o8 = out[warp] + 8 * lane;
  packed = make_uint4(pack_bf2(o8[0], o8[1]), pack_bf2(o8[2], o8[3]), pack_bf2(o8[4], o8[5]),
                      pack_bf2(o8[6], o8[7]));
  if (warp < 8) {
    *reinterpret_cast<uint4*>(a.qn + (size_t(warp) * a.tmax + t) * 256 + 8 * lane) = packed;
  } else {
    const int kh = warp - 8;
    const uint32_t p = a.p0 + uint32_t(t), cps = a.capacity / kAttnChains;
    const size_t ci = (size_t(kh) * a.capacity + size_t(p % kAttnChains) * cps + p / kAttnChains) * 256;
    *reinterpret_cast<uint4*>(a.kcache + ci + 8 * lane) = packed;
    *reinterpret_cast<uint4*>(a.vcache + ci + 8 * lane) =
        *reinterpret_cast<const uint4*>(a.v_raw + size_t(t) * 512 + kh * 256 + 8 * lane);
  }
}

// Flash attention work item = (KV head, 32-token query block, key split):
// rows r = 32 hq + i (query head 4 kvh + hq, token 32 qb + i), keys in 64-key
// tiles [tb, te) of the split. Two launches: PASS 0 computes S = Q K^T over
// the split and each row's maximum; PASS 1 takes the row maximum M over all
// splits, recomputes S and accumulates O += P V with P = bf16(e^((S - M) / 16))
// (pa_weight), so every split weighs its keys against the same maximum
// (the combine then only adds). Roles: warp 0 lane 0 loads Q once and the key
// and value tiles through a ring (3-D TMA, 128-byte swizzle), warp 1 lane 0
// issues the MMAs, warp 2 owns the TMEM allocation, warps 4-7 (thread = row =
// TMEM lane) read S, form P and drain O. TMEM: S in two 64-column buffers, O
// in columns 256..511.
constexpr int kPaStages = 3;
constexpr uint32_t kPaQBytes = 128 * 256 * 2;    // Q: 4 swizzled 64-dim blocks of 128 rows
constexpr uint32_t kPaTileBytes = 64 * 256 * 2;  // one key or value tile: 4 blocks of 64 keys x 64 dims
constexpr uint32_t kPaPBytes = 128 * 64 * 2;     // P: 128 rows x 64 keys
constexpr size_t kPaSmem = 1024 + kPaQBytes + kPaStages * kPaTileBytes + 2 * kPaPBytes + 256;
// exp(x / 16) = 2^(x log2(e) / 16): the 1/sqrt(256) score scale folded in
// (the combine's split factors, which are all 1: every split carries the
// row's maximum)
constexpr float kPaExp2Scale = 0.0901684400555602f;

// The attention weight of a score s against the row maximum m:
// e^((s - m) / 16) by the decode kernels' fexp (Cody-Waite reduction and a
// polynomial of IEEE-exact operations, so the CPU oracle restates it bit for
// bit), rounded to bf16 by the caller.
Q35_DEV float pa_weight(float s, float m) { return fexp(__fmul_rn(__fsub_rn(s, m), 0.0625f)); }

Q35_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

template <int PASS>
__global__ void __launch_bounds__(256, 1) k_pr_attn(const __grid_constant__ PromptArgs a) {
  extern __shared__ uint8_t dsm[];
  const uint32_t base_u = smem_u32(dsm);
  uint8_t* sm = dsm + (((base_u + 1023u) & ~1023u) - base_u);  // swizzled tiles: 1024-byte aligned
  uint8_t* Qs = sm;
  uint8_t* Ring = Qs + kPaQBytes;
  uint8_t* Ps = Ring + kPaStages * kPaTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(Ps + 2 * kPaPBytes);
  uint64_t* qfull = bars;
  uint64_t* kvfull = bars + 1;
  uint64_t* kvempty = kvfull + kPaStages;
  uint64_t* sfull = kvempty + kPaStages;
  uint64_t* sfree = sfull + 2;
  uint64_t* pfull = sfree + 2;
  uint64_t* pfree = pfull + 2;
  uint64_t* ofull = pfree + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(ofull + 1);
  volatile int* bad = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTAs in launch order walk the query blocks innermost, so the CTAs resident
  // together read the same key range (served from L2); partials are indexed
  // by (KV head, query block, split)
  const int qb = blockIdx.x % a.nqb, rest = blockIdx.x / a.nqb;
  const int sp = rest % a.nsplit, kvh = rest / a.nsplit;
  const int pair = kvh * a.nqb + qb, item = pair * a.nsplit + sp;
  const int qlast = min(a.T, qb * 32 + 32) - 1;
  const int ntile = int((a.p0 + uint32_t(qlast)) / 64u) + 1;  // key tiles the block reaches
  const int tb = int(int64_t(ntile) * sp / a.nsplit), te = int(int64_t(ntile) * (sp + 1) / a.nsplit);
  const int n = te - tb;
  float* opart = a.opart + size_t(item) * 128 * 256;
  float* oml = a.oml + size_t(item) * 128 * 2;
  const int nseq = PASS == 0 ? n : 2 * n;  // ring elements of this pass

  if (warp == 2) tc_alloc(tslot, 512);
  if (tid == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < kPaStages; ++s) {
      mbar_init(&kvfull[s], 1);
      mbar_init(&kvempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&sfree[b], 4);
      mbar_init(&pfull[b], 4);
      mbar_init(&pfree[b], 1);
    }
    mbar_init(ofull, 1);
    *bad = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();  // queries and the cache come from the previous launch
  pdl_launch();
  auto wait = [&](uint64_t* b, uint32_t parity) {
    if (*bad) return false;
    if (!mbar_wait(b, parity, a.ctl, kErrPromptWait)) {
      *bad = 1;
      return false;
    }
    return true;
  };
  // ring sequence: PASS 0 K_0 .. K_{n-1}; PASS 1 K_0, then (K_{j+1}, V_j) for
  // j < n - 1, then V_{n-1} (the MMA computes S_{j+1} before O += P_j V_j)
  auto seq_elem = [&](int g, bool& is_v, int& j) {
    if (PASS == 0) {
      is_v = false;
      j = g;
      return;
    }
    const int h = g;
    if (h == 0) {
      is_v = false;
      j = 0;
      return;
    }
    const int q = h - 1, jj = q >> 1;
    if (jj < n - 1) {
      is_v = (q & 1) != 0;
      j = is_v ? jj : jj + 1;
    } else {
      is_v = true;
      j = n - 1;
    }
  };

  if (warp == 0 && lane == 0 && n > 0) {
    // ---------------- loader ----------------
    mbar_expect_tx(qfull, kPaQBytes);
    for (int kb = 0; kb < 4; ++kb) tma_load_3d(Qs + kb * 16384, &a.qmap, kb * 64, qb * 32, kvh * 4, qfull);
    for (int g = 0; g < nseq; ++g) {
      const int s = g % kPaStages, u = g / kPaStages;
      if (u >= 1 && !wait(&kvempty[s], uint32_t(u - 1) & 1u)) break;
      bool is_v;
      int j;
      seq_elem(g, is_v, j);
      mbar_expect_tx(&kvfull[s], kPaTileBytes);
      for (int kb = 0; kb < 4; ++kb)
        tma_load_3d(Ring + s * kPaTileBytes + kb * 8192, is_v ? &a.vmap : &a.kmap, kb * 64, tb + j, kvh * 64,
                    &kvfull[s]);
    }
  } else if (warp == 1 && lane == 0 && n > 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t id_s = tc_idesc_bf16(128, 64);
    const uint32_t id_o = tc_idesc_bf16(128, 256) | (1u << 16);  // B (the value tile) MN-major
    int g = 0, u = 0;
    auto mma_s = [&]() -> bool {  // S[u % 2] = Q K^T, K = ring element g
      const int s = g % kPaStages;
      if (!wait(&kvfull[s], uint32_t(g / kPaStages) & 1u)) return false;
      if (u >= 2 && !wait(&sfree[u & 1], uint32_t((u >> 1) - 1) & 1u)) return false;
      tc_fence_after();
      const uint32_t d = tmem + uint32_t((u & 1) * 64);
      const uint32_t q0 = smem_u32(Qs), k0 = smem_u32(Ring + s * kPaTileBytes);
#pragma unroll
      for (int kb = 0; kb < 4; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(d, tc_desc_sw128(q0 + kb * 16384 + kk * 32, 1024), tc_desc_sw128(k0 + kb * 8192 + kk * 32, 1024),
                      id_s, (kb | kk) ? 1u : 0u);
      tc_commit(&kvempty[s]);
      tc_commit(&sfull[u & 1]);
      ++g;
      ++u;
      return true;
    };
    bool ok = wait(qfull, 0);
    if (PASS == 0) {
      for (int j = 0; j < n && ok; ++j) ok = mma_s();
    } else if (ok) {
      ok = mma_s();  // S_0
    }
    for (int j = 0; j < n && ok && PASS == 1; ++j) {
      if (j + 1 < n && !(ok = mma_s())) break;
      const int s = g % kPaStages;
      if (!(ok = wait(&kvfull[s], uint32_t(g / kPaStages) & 1u))) break;
      if (!(ok = wait(&pfull[j & 1], uint32_t(j >> 1) & 1u))) break;
      tc_fence_after();
      const uint32_t pa = smem_u32(Ps + (j & 1) * kPaPBytes), v0 = smem_u32(Ring + s * kPaTileBytes);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc_mma_bf16(tmem + 256, tc_desc_sw128(pa + kk * 32, 1024), tc_desc_sw128_mn(v0 + kk * 2048, 8192, 1024),
                    id_o, (j | kk) ? 1u : 0u);
      tc_commit(&kvempty[s]);
      tc_commit(&pfree[j & 1]);
      ++g;
    }
    if (ok && PASS == 1) tc_commit(ofull);
  } else if (warp >= 4) {
    // ---------------- softmax / output ----------------
    const int e = tid - 128;  // row = TMEM lane
    const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
    const int64_t rowpos = int64_t(a.p0) + qb * 32 + (e & 31);
    float m = -INFINITY, l = 0.0f;
    int u = 0;
    float sv[64];
    auto load_s = [&]() -> bool {
      if (!wait(&sfull[u & 1], uint32_t(u >> 1) & 1u)) return false;
      tc_fence_after();
      tc_ld32(tmem + lane_base + uint32_t((u & 1) * 64), sv);
      tc_ld32(tmem + lane_base + uint32_t((u & 1) * 64 + 32), sv + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[u & 1]);
      ++u;
      return true;
    };
    bool ok = true;
    if (PASS == 0) {
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = -INFINITY;
      for (int j = 0; j < n && ok; ++j) {
        if (!(ok = load_s())) break;
        const int64_t k0 = int64_t(tb + j) * 64;
        if (k0 + 63 <= rowpos) {
#pragma unroll
          for (int c = 0; c < 64; ++c) mp[c & 7] = fmaxf(mp[c & 7], sv[c]);
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (k0 + c <= rowpos) mp[c & 7] = fmaxf(mp[c & 7], sv[c]);
        }
      }
      m = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      if (ok) a.omax[size_t(item) * 128 + e] = m;  // -inf for an empty split
    } else {
      const float* om = a.omax + size_t(pair) * a.nsplit * 128 + e;
      for (int s2 = 0; s2 < a.nsplit; ++s2) m = fmaxf(m, __ldcg(om + size_t(s2) * 128));
    }
    float lp[8];  // partial sums of the bf16 weights
#pragma unroll
    for (int i = 0; i < 8; ++i) lp[i] = 0.0f;
    for (int j = 0; j < n && ok && PASS == 1; ++j) {
      if (!(ok = load_s())) break;
      const int64_t k0 = int64_t(tb + j) * 64;
      const bool diag = k0 + 63 > rowpos;  // only tiles reaching past the row's position are masked
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        float x0 = pa_weight(sv[c], m);
        float x1 = pa_weight(sv[c + 1], m);
        if (diag) {
          if (k0 + c > rowpos) x0 = 0.0f;
          if (k0 + c + 1 > rowpos) x1 = 0.0f;
        }
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(x0, x1);
        const uint32_t w = *reinterpret_cast<const uint32_t*>(&p2);
        pk[c >> 1] = w;
        lp[(c >> 1) & 7] = __fadd_rn(lp[(c >> 1) & 7], __fadd_rn(bf_lo(w), bf_hi(w)));
      }
      if (j >= 2 && !(ok = wait(&pfree[j & 1], uint32_t((j >> 1) - 1) & 1u))) break;
      uint8_t* P = Ps + (j & 1) * kPaPBytes;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(P + sw128_off(e, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[j & 1]);
    }
    if (PASS == 0) {
    } else if (n == 0) {
      oml[e * 2] = -INFINITY;  // an empty split: no weight in the combine
      oml[e * 2 + 1] = 0.0f;
    } else if (ok && wait(ofull, 0)) {
      l = __fadd_rn(__fadd_rn(__fadd_rn(lp[0], lp[1]), __fadd_rn(lp[2], lp[3])),
                    __fadd_rn(__fadd_rn(lp[4], lp[5]), __fadd_rn(lp[6], lp[7])));
      tc_fence_after();
      float* orow = opart + size_t(e) * 256;
      for (int c0 = 0; c0 < 256; c0 += 32) {
        float ov[32];
        tc_ld32(tmem + lane_base + 256 + uint32_t(c0), ov);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(orow + c0 + i) = make_float4(ov[i], ov[i + 1], ov[i + 2], ov[i + 3]);
      }
      oml[e * 2] = m;
      oml[e * 2 + 1] = l;
    }
  }
  __syncwarp();  // the loader and MMA lanes rejoin their warps
  tc_fence_before();
  __syncthreads();
  if (warp == 2) tc_dealloc(tmem, 512);
}

// grid (T, 8 query heads) x 256 dims: out = sum_s f_s O_s / sum_s f_s l_s with
// f_s = exp((m_s - M) / 16), M the largest split maximum (every split of a row
// carries the same maximum, so f_s = 1 and the sums run in split order); then
// the gate.
__global__ void __launch_bounds__(256) k_pr_attn_combine(const __grid_constant__ PromptArgs a) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x, qh = blockIdx.y, d = threadIdx.x;
  const int kvh = qh >> 2, e = (qh & 3) * 32 + (t & 31);
  const size_t item0 = (size_t(kvh) * a.nqb + (t >> 5)) * a.nsplit;
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, __ldcg(&a.oml[((item0 + s) * 128 + e) * 2]));
  float L = 0.0f, O = 0.0f;
  for (int s = 0; s < a.nsplit; ++s) {
    const float ms = __ldcg(&a.oml[((item0 + s) * 128 + e) * 2]);
    if (ms == -INFINITY) continue;
    const float f = exp2f(__fmul_rn(__fsub_rn(ms, M), kPaExp2Scale));
    L = __fadd_rn(L, __fmul_rn(f, __ldcg(&a.oml[((item0 + s) * 128 + e) * 2 + 1])));
    O = __fadd_rn(O, __fmul_rn(f, __ldcg(&a.opart[((item0 + s) * 128 + e) * 256 + d])));
  }
  const float attention = bfr(__fdiv_rn(O, L));
  a.gated[size_t(t) * 2048 + qh * 256 + d] =
      f2bf(__fmul_rn(attention, attn_gate_bf(bf2f(a.q_raw[size_t(t) * kQProj + qh * 512 + 256 + d]))));
}

// RoPE rows of positions p0 .. p0 + T - 1 (the standalone attention op; in a
// prompt chunk the first layer's embedding kernel records them).
__global__ void __launch_bounds__(32) k_pr_rope(uint32_t p0, float* rope) {
  pdl_wait();
  pdl_launch();
  rope_pair(p0 + blockIdx.x, threadIdx.x, rope + 64 * blockIdx.x);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
cudaError_t prompt_kernels_init() {
  cudaError_t e = cudaFuncSetAttribute(k_pr_recur, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPrRecSmem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_pr_attn<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPaSmem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_pr_attn<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kPaSmem));
  return e;
}

// Key splits: enough items for ~3 CTAs per SM, at most 128 tiles (8192 keys)
// per split, never more splits than tiles.
static int attn_splits(int nqb, int maxtiles) {
  const int want = (444 + 2 * nqb - 1) / (2 * nqb);
  int ns = (maxtiles + 127) / 128;
  if (ns < want) ns = want;
  if (ns > maxtiles) ns = maxtiles;
  return ns < 1 ? 1 : ns;
}

size_t prompt_attn_items_max(int tmax, uint32_t capacity) {
  const int nqb = tmax / 32;
  const size_t a = 444 + 2 * size_t(nqb), b = 2 * size_t(nqb) * ((capacity + 8191) / 8192);
  return a > b ? a : b;
}

void prompt_attn_plan(PromptArgs& a) {
  a.nqb = (a.T + 31) / 32;
  const int maxtiles = int((a.p0 + uint32_t(a.T) - 1) / 64u) + 1;
  a.nsplit = attn_splits(a.nqb, maxtiles);
}

cudaError_t launch_prompt_rope(uint32_t p0, int T, float* rope, cudaStream_t st, bool pdl) {
  return launch_ex(k_pr_rope, dim3(T), dim3(32), 0, st, pdl, p0, rope);
}
cudaError_t launch_prompt_conv(const PromptArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_pr_conv, dim3(kGdnConv / 512, (a.T + kPrConvTokens - 1) / kPrConvTokens), dim3(256), 0, st,
                   pdl, a);
}
cudaError_t launch_prompt_gdn_prep(const PromptArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_pr_gdn_prep, dim3(a.T), dim3(512), 0, st, pdl, a);
}
cudaError_t launch_prompt_recur(const PromptArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_pr_recur, dim3(8, kGdnHeads), dim3(128), kPrRecSmem, st, pdl, a);
}
cudaError_t launch_prompt_attn_prep(const PromptArgs& a, cudaStream_t st, bool pdl) {
  return launch_ex(k_pr_attn_prep, dim3(a.T), dim3(320), 0, st, pdl, a);
}

// Encodes the query/key/value descriptors, then the attention items and the
// combine. The key/value maps cover the layer's whole cache (capacity / 64
// slots per chain).
cudaError_t launch_prompt_attn(PromptArgs a, cudaStream_t st, bool pdl) {
  if (a.T < 1 || a.T > a.tmax || a.capacity % kAttnChains != 0 || a.nqb != (a.T + 31) / 32 || a.nsplit < 1)
    return cudaErrorInvalidValue;
  const uint64_t cps = a.capacity / kAttnChains;
  if (!tmap_3d(&a.qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.qn, 256, uint64_t(a.T), 8, 512,
               uint64_t(a.tmax) * 512, 64, 32, 4, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap_3d(&a.kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.kcache, 256, cps, 2 * kAttnChains, 512, cps * 512, 64,
               1, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap_3d(&a.vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.vcache, 256, cps, 2 * kAttnChains, 512, cps * 512, 64,
               1, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const int items = 2 * a.nqb * a.nsplit;
  cudaError_t e = launch_ex(k_pr_attn<0>, dim3(items), dim3(256), kPaSmem, st, pdl, a);
  if (e == cudaSuccess) e = launch_ex(k_pr_attn<1>, dim3(items), dim3(256), kPaSmem, st, true, a);
  if (e != cudaSuccess) return e;
  return launch_ex(k_pr_attn_combine, dim3(a.T, 8), dim3(256), 0, st, true, a);
}

}  // namespace q35
