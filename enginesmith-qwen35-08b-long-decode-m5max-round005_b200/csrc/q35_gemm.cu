// Q4 affine GEMM on the 5th-generation tensor cores, for batched sessions:
// y[t][n] = bf16(sum_k W[n][k] x[t][k]) for T tokens at once, with W the
// MLX affine Q4 matrix dequantised as bf16(s q + b) (the reference's
// quantised-matmul route dequantises to the activation type, linear_nax.metal
// qmm_q4_nax). Unlike the exact matvec this changes the summation order, so it
// matches a float32 reference within tolerance, not bit for bit.
//
// Swap-AB tiling: the 128 weight rows of a CTA are the MMA's M, the tokens
// its N (16..256), K runs in blocks of 64 (one quantisation group, so one
// scale/bias per row and block). Per block two threads dequantise one row's
// 64 weights into shared memory in the 128-byte-swizzled K-major layout, the
// tokens' activations are stored beside them in the same layout, and one
// thread issues four 128 x Np x 16 MMAs accumulating in TMEM; two
// shared-memory stages let the next block's dequantisation overlap the
// running MMAs (tcgen05.commit to a per-stage mbarrier). A CTA's codes,
// scales and biases arrive by bulk copy (the next work item's behind the
// current epilogue); CTAs are persistent over (row tile, K split) items, and
// the last CTA of a split tile sums the f32 partials in split order
// (deterministic). The epilogue reads TMEM with tcgen05.ld (thread = row, 8
// tokens per load).
#include <cuda_runtime.h>

#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_tc.cuh"
#include "q35_types.h"

namespace q35 {


constexpr int kGemmRows = 128;
constexpr int kGemmKb = 64;
constexpr int kGemmThreads = 512;  // four per weight row
constexpr int kGemmQuarters = kGemmThreads / 128;
constexpr int kGemmMaxTokens = 256;
constexpr int kGemmMaxKb = 16;  // K blocks per work item (its codes are staged whole)
constexpr uint32_t kErrGemmWait = 8;
// The workspace starts with the split counters (kGemmMaxTiles words, then the
// error word) at a fixed offset, so GEMMs of different shapes can share one
// workspace: every counter is zero between launches (the last CTA of a split
// tile resets its own), whatever the other GEMMs left in the partials.
constexpr int kGemmMaxTiles = 4096;
constexpr size_t kGemmCounterBytes = size_t(kGemmMaxTiles) * 4 + 256;

__host__ __device__ inline int gemm_np(int T) { return ((T + 15) / 16) * 16; }
__host__ __device__ inline size_t gemm_a_bytes() { return size_t(kGemmRows) * kGemmKb * 2; }
__host__ __device__ inline size_t gemm_b_bytes(int Np) { return size_t(Np) * kGemmKb * 2; }
// a row's staged codes: kblocks x 32 bytes plus 16 bytes of padding, so
// consecutive rows fall on different banks
__host__ __device__ inline int gemm_code_stride(int kblocks) { return kblocks * 32 + 16; }
struct GemmLayout {
  size_t a, b, codes, scl, bia, bar, total;
};
__host__ __device__ inline GemmLayout gemm_layout(int Np, int kblocks, int K) {
  GemmLayout L;
  L.a = 0;
  L.b = L.a + 2 * gemm_a_bytes();
  L.codes = L.b + 2 * gemm_b_bytes(Np);
  L.scl = L.codes + size_t(kGemmRows) * gemm_code_stride(kblocks);
  L.bia = L.scl + size_t(kGemmRows) * (K / 64) * 2;
  L.bar = (L.bia + size_t(kGemmRows) * (K / 64) * 2 + 15) & ~size_t(15);
  L.total = L.bar + 64;
  return L;
}
__host__ __device__ inline uint32_t gemm_tmem_cols(int Np) {
  uint32_t c = 32;
  while (c < uint32_t(Np)) c <<= 1;
  return c;
}

// Persistent: CTA c takes work items c, c + gridDim.x, ... of the
// (row tile, K split) grid `tiles x splits` (item = tile * splits + split).
// The segment of global row tile `tile`, its first tile and its first row in
// the concatenated row space.
__device__ __forceinline__ int gemm_seg_of(const QGemmArgs& a, int tile, int* tile0, int* grow0) {
  int t0 = 0, r0 = 0;
#pragma unroll
  for (int i = 0; i < kGemmSegs; ++i) {
    const int nt = (a.seg[i].rows + kGemmRows - 1) / kGemmRows;
    if (i == a.nseg - 1 || tile < t0 + nt) {
      *tile0 = t0;
      *grow0 = r0;
      return i;
    }
    t0 += nt;
    r0 += a.seg[i].rows;
  }
  return 0;
}

__global__ void __launch_bounds__(kGemmThreads, 1) k_qgemm(const __grid_constant__ QGemmArgs a) {
  const int tiles = a.tiles, splits = a.splits;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ int last;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int K = a.K, KW = K / 8, KG = K / 64, nkb = K / kGemmKb;
  const int T = a.T, Np = a.Np;
  const GemmLayout L = gemm_layout(Np, a.kblocks, K);
  uint8_t* As = smem + L.a;
  uint8_t* Bs = smem + L.b;
  uint8_t* codes = smem + L.codes;
  const uint16_t* scl = reinterpret_cast<const uint16_t*>(smem + L.scl);
  const uint16_t* bia = reinterpret_cast<const uint16_t*>(smem + L.bia);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);  // [0,1] MMA stages, [2] weights
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 3);
  int* bad = reinterpret_cast<int*>(tslot + 1);
  const uint32_t cols = gemm_tmem_cols(Np);
  const int nitems = tiles * splits;
  const int r = tid & (kGemmRows - 1), qtr = tid >> 7;  // row, quarter of its 64 values

  if (warp == 0) tc_alloc(tslot, cols);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
    // the swizzled operand tiles need 1024-byte aligned bases
    *bad = (smem_u32(smem) & 1023u) != 0u;
    if (*bad && a.err) atomicCAS(a.err, 0u, kErrGemmWait);
  }
  for (int i = tid; i < 2 * (Np - T) * 8; i += kGemmThreads) {  // padding tokens stay zero
    const int s = i / ((Np - T) * 8), q = i % ((Np - T) * 8), t = T + q / 8, j = q % 8;
    *reinterpret_cast<uint4*>(Bs + s * gemm_b_bytes(Np) + sw128_off(t, j)) = make_uint4(0u, 0u, 0u, 0u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // stage an item's weights: the codes of its K blocks (one bulk copy per
  // row) and its tile's scales and biases (one copy each)
  auto stage = [&](int item) {
    const int tile = item / splits, sp = item - tile * splits;
    int stile0, sgrow0;
    const QGemmSeg& sg = a.seg[gemm_seg_of(a, tile, &stile0, &sgrow0)];
    const int row0 = (tile - stile0) * kGemmRows, nrows = min(kGemmRows, sg.rows - row0);
    const int kb0 = sp * a.kblocks, nit = min(nkb, kb0 + a.kblocks) - kb0;
    fence_proxy_async();  // earlier generic reads of these buffers before the copies
    if (tid == 0) {
      const uint32_t sb = uint32_t(nrows) * KG * 2;
      mbar_expect_tx(&bar[2], uint32_t(nrows) * nit * 32 + 2 * sb);
      bulk_g2s(smem + L.scl, sg.s + size_t(row0) * KG, sb, &bar[2]);
      bulk_g2s(smem + L.bia, sg.b + size_t(row0) * KG, sb, &bar[2]);
    }
    __syncthreads();  // expect_tx is registered before any code copy lands
    if (tid < nrows)
      bulk_g2s(codes + tid * gemm_code_stride(a.kblocks), sg.w + size_t(row0 + tid) * KW + size_t(kb0) * 8,
               uint32_t(nit) * 32, &bar[2]);
  };
  if (int(blockIdx.x) < nitems) stage(blockIdx.x);
  pdl_wait();
  pdl_launch();

  constexpr int kBRegs = kGemmMaxTokens * 8 / kGemmThreads;
  uint4 breg[kBRegs];
  // activations of block kb: element i = j * T + t (token fastest, so the
  // shared-memory stores of 8 consecutive threads are one 128-byte row);
  // each slot's source offset and tile offset are fixed for the kernel
  size_t bsrc[kBRegs];
  uint32_t bdst[kBRegs];
#pragma unroll
  for (int q = 0; q < kBRegs; ++q) {
    const int i = tid + q * kGemmThreads, j = i / T, t = i - j * T;
    bsrc[q] = size_t(t) * K + size_t(j) * 8;
    bdst[q] = sw128_off(t, j);
  }
  auto load_b = [&](int kb) {
#pragma unroll
    for (int q = 0; q < kBRegs; ++q)
      if (tid + q * kGemmThreads < T * 8)
        breg[q] = __ldg(reinterpret_cast<const uint4*>(a.x + bsrc[q] + size_t(kb) * kGemmKb));
  };
  const uint32_t idesc = tc_idesc_bf16(kGemmRows, Np);
  const uint32_t tbase = tmem + (uint32_t(32 * (warp & 3)) << 16);
  uint32_t wphase = 0, mma_uses[2] = {0u, 0u};

  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const int tile = item / splits, sp = item - tile * splits;
    int stile0, sgrow0;
    const QGemmSeg& sg = a.seg[gemm_seg_of(a, tile, &stile0, &sgrow0)];
    const int row0 = (tile - stile0) * kGemmRows, nrows = min(kGemmRows, sg.rows - row0);
    const int kb0 = sp * a.kblocks, nit = min(nkb, kb0 + a.kblocks) - kb0;
    const bool rok = r < nrows;
    const int row = row0 + r;              // row within the segment
    const int grow = sgrow0 + row;         // row in the concatenated space (partials)
    // CTAs walk their K blocks from different starting blocks, so they do
    // not all read the same activation lines at the same moment
    const int rot = nit > 0 ? int(blockIdx.x) % nit : 0;
    load_b(kb0 + rot);
    if (!mbar_wait_limit(&bar[2], wphase, kWaitLimit, a.err, kErrGemmWait)) *bad = 1;
    wphase ^= 1u;
    const uint8_t* crow = codes + r * gemm_code_stride(a.kblocks) + qtr * 8;
    for (int it = 0; it < nit; ++it) {
      const int ib = it + rot < nit ? it + rot : it + rot - nit;  // block within the item
      const int kb = kb0 + ib, s = it & 1;
      if (mma_uses[s] > 0 &&
          !mbar_wait_limit(&bar[s], (mma_uses[s] - 1) & 1u, kWaitLimit, a.err, kErrGemmWait))
        *bad = 1;
      uint8_t* A = As + s * gemm_a_bytes();
      uint8_t* B = Bs + s * gemm_b_bytes(Np);
#pragma unroll
      for (int q = 0; q < kBRegs; ++q)
        if (tid + q * kGemmThreads < T * 8) *reinterpret_cast<uint4*>(B + bdst[q]) = breg[q];
      if (it + 1 < nit) load_b(kb0 + (ib + 1 < nit ? ib + 1 : 0));
      // this thread's 32 of its row's 64 values -> bf16(s q + b), 4 core matrices
      uint2 c = make_uint2(0u, 0u);
      float sc = 0.0f, bi = 0.0f;
      if (rok) {
        c = *reinterpret_cast<const uint2*>(crow + ib * 32);
        sc = bf2f(scl[r * KG + kb]);
        bi = bf2f(bia[r * KG + kb]);
      }
      const uint32_t words[2] = {c.x, c.y};
      // packed bf16: the nibbles at word positions (e, e + 4) become the pair
      // (128 + n_e, 128 + n_{e+4}) by one LOP3 with the bf16 bits of 128; an
      // exact subtraction of 128 and one fma rounding to nearest even give
      // bf16(s q + b) (s q is exact, so this is the correctly rounded value),
      // and byte permutes restore the order (0,1) (2,3) (4,5) (6,7)
      const __nv_bfloat162 s2 = __floats2bfloat162_rn(sc, sc), b2 = __floats2bfloat162_rn(bi, bi);
      const __nv_bfloat162 m128 = __floats2bfloat162_rn(128.0f, 128.0f);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t m = ((words[j] >> (4 * e)) & 0x000f000fu) | 0x43004300u;  // nibbles e, e + 4
          const __nv_bfloat162 q2 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&m), m128);
          const __nv_bfloat162 w2 = __hfma2(s2, q2, b2);
          v[e] = *reinterpret_cast<const uint32_t*>(&w2);  // lo: value e, hi: value e + 4
        }
        const uint4 o = rok ? make_uint4(__byte_perm(v[0], v[1], 0x5410), __byte_perm(v[2], v[3], 0x5410),
                                         __byte_perm(v[0], v[1], 0x7632), __byte_perm(v[2], v[3], 0x7632))
                            : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(A + sw128_off(r, qtr * 2 + j)) = o;
      }
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      if (tid == 0 && !*bad) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(tmem, tc_desc_sw128(a0 + 32 * kk, 1024), tc_desc_sw128(b0 + 32 * kk, 1024), idesc,
                      (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&bar[s]);
      }
      ++mma_uses[s];
    }
    // every code of this item is read: stage the next item behind the epilogue
    const int next = item + int(gridDim.x);
    if (next < nitems) stage(next);
    const int sl = (nit - 1) & 1;
    if (nit > 0 && !mbar_wait_limit(&bar[sl], (mma_uses[sl] - 1) & 1u, kWaitLimit, a.err, kErrGemmWait))
      *bad = 1;
    tc_fence_after();
    const bool ok = !*bad && nit > 0;
    const bool splitk = splits > 1;
    if (ok) {
      // warp w reads TMEM lanes 32 (w % 4).. and token part w / 4 (8-token units)
      const int tph = ((T + 8 * kGemmQuarters - 1) / (8 * kGemmQuarters)) * 8;
      const int c0 = (warp >> 2) * tph, c1 = min(T, c0 + tph);
      for (int cc = c0; cc < c1; cc += 8) {
        float v[8];
        tc_ld8(tbase + uint32_t(cc), v);
        if (!rok) continue;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int t = cc + e;
          if (t >= c1) break;
          if (splitk) {
            a.part[(size_t(sp) * T + t) * a.rows_total + grow] = v[e];
          } else {
            uint16_t* y = sg.y + size_t(t) * sg.ystride + row;
            if (sg.res)
              *y = f2bf(__fadd_rn(bf2f(sg.res[size_t(t) * sg.ystride + row]), bfr(v[e])));
            else
              *y = f2bf(v[e]);
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM reads done before the next item's first MMA
    if (!splitk || !ok) continue;

    // split K: the last CTA of this row tile sums the partials in split order
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&a.counters[tile], 1u) == uint32_t(splits - 1);
    __syncthreads();
    if (!last) continue;
    __threadfence();
    if (tid == 0) a.counters[tile] = 0;
    if (rok) {
      for (int t0 = qtr * 8; t0 < T; t0 += 8 * kGemmQuarters) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
        for (int q = 0; q < splits; ++q) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (t0 + e < T) acc[e] = __fadd_rn(acc[e], __ldcg(&a.part[(size_t(q) * T + t0 + e) * a.rows_total + grow]));
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int t = t0 + e;
          if (t >= T) break;
          uint16_t* y = sg.y + size_t(t) * sg.ystride + row;
          if (sg.res)
            *y = f2bf(__fadd_rn(bf2f(sg.res[size_t(t) * sg.ystride + row]), bfr(acc[e])));
          else
            *y = f2bf(acc[e]);
        }
      }
    }
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tc_dealloc(tmem, cols);
}

// Host side ------------------------------------------------------------------
static int gemm_tiles(const QGemmArgs& a) {
  int t = 0;
  for (int i = 0; i < a.nseg; ++i) t += (a.seg[i].rows + kGemmRows - 1) / kGemmRows;
  return t;
}
static int gemm_rows(const QGemmArgs& a) {
  int r = 0;
  for (int i = 0; i < a.nseg; ++i) r += a.seg[i].rows;
  return r;
}

void qgemm_plan(int tiles, int K, int* splits, int* kblocks) {
  const int nkb = K / kGemmKb > 0 ? K / kGemmKb : 1;
  int sp = (148 + tiles - 1) / tiles;
  if (sp > nkb) sp = nkb;
  if (sp < (nkb + kGemmMaxKb - 1) / kGemmMaxKb) sp = (nkb + kGemmMaxKb - 1) / kGemmMaxKb;
  if (sp < 1) sp = 1;
  const int kb = (nkb + sp - 1) / sp;
  *kblocks = kb;
  *splits = (nkb + kb - 1) / kb;
}

size_t qgemm_workspace_bytes(const QGemmArgs& a) {
  const int tiles = gemm_tiles(a);
  int splits, kb;
  qgemm_plan(tiles, a.K, &splits, &kb);
  const size_t part = splits > 1 ? size_t(splits) * a.T * gemm_rows(a) * 4 : 0;
  return kGemmCounterBytes + part;
}

size_t qgemm_workspace_bytes(int N, int K, int T) {
  QGemmArgs a = {};
  a.nseg = 1;
  a.seg[0].rows = N;
  a.K = K;
  a.T = T;
  return qgemm_workspace_bytes(a);
}

cudaError_t qgemm_init() {
  return cudaFuncSetAttribute(k_qgemm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(gemm_layout(kGemmMaxTokens, kGemmMaxKb, 4096).total));
}

// Validates, lays out the workspace (partials, counters, error word) and
// launches. The counters must be zero; `zero_counters` clears them first.
cudaError_t launch_qgemm(QGemmArgs a, void* ws, size_t ws_bytes, bool zero_counters, cudaStream_t st, bool pdl) {
  if (a.T < 1 || a.T > kGemmMaxTokens || a.K % 512 != 0 || a.K < 512 || a.K > 4096 || a.nseg < 1 ||
      a.nseg > kGemmSegs || !a.x)
    return cudaErrorInvalidValue;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].rows < 1 || !a.seg[i].w || !a.seg[i].s || !a.seg[i].b || !a.seg[i].y ||
        a.seg[i].ystride < a.seg[i].rows)
      return cudaErrorInvalidValue;
  if (ws_bytes < qgemm_workspace_bytes(a)) return cudaErrorInvalidValue;
  const int tiles = gemm_tiles(a);
  if (tiles > kGemmMaxTiles) return cudaErrorInvalidValue;
  int splits, kb;
  qgemm_plan(tiles, a.K, &splits, &kb);
  a.tiles = tiles;
  a.splits = splits;
  a.kblocks = kb;
  a.rows_total = gemm_rows(a);
  uint8_t* w = static_cast<uint8_t*>(ws);
  a.counters = reinterpret_cast<uint32_t*>(w);
  a.part = reinterpret_cast<float*>(w + kGemmCounterBytes);
  if (!a.err) a.err = a.counters + kGemmMaxTiles;
  a.Np = gemm_np(a.T);
  if (zero_counters) {
    cudaError_t e = cudaMemsetAsync(a.counters, 0, kGemmCounterBytes, st);
    if (e != cudaSuccess) return e;
  }
  const int items = tiles * splits;
  const int grid = items < 148 ? items : 148;
  return launch_ex(k_qgemm, dim3(grid), dim3(kGemmThreads), gemm_layout(a.Np, kb, a.K).total, st, pdl, a);
}

}  // namespace q35
