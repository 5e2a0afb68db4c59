// Q4 affine GEMM on the 5th-generation tensor cores, for batched sessions:
// y[t][n] = bf16(sum_k W[n][k] x[t][k]) for T tokens at once, with W the
// MLX affine Q4 matrix dequantised as bf16(s q + b) (the reference's
// quantised-matmul route dequantises to the activation type, linear_nax.metal
// qmm_q4_nax). Unlike the exact matvec this changes the summation order, so it
// matches a float32 reference within tolerance, not bit for bit.
//
// Swap-AB tiling: the 128 weight rows of a CTA are the MMA's M, a tile of up
// to 256 tokens its N (16..256), K runs in blocks of 64 (one quantisation
// group, so one scale/bias per row and block). A persistent CTA walks (row
// tile, token tile, K split) work items with warp-specialised roles linked by mbarriers: a loader thread
// brings each block's codes and the tokens' activations in by 2-D TMA (the
// activations already in the 128-byte-swizzled K-major layout) and each item's
// scales and biases by bulk copy; eight producer warps dequantise the block
// (packed bf16) into the same swizzled layout; one thread issues four
// 128 x Np x 16 MMAs per block into one of two TMEM accumulators
// (tcgen05.commit frees the stage); four epilogue warps drain the other
// accumulator with tcgen05.ld while the next item accumulates. A ring of 2-4
// stages decouples the roles. Split partials (f32) are summed in split order
// by a second kernel (deterministic).
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "q35_kernels.h"
#include "q35_launch.h"
#include "q35_tc.cuh"
#include "q35_types.h"

namespace q35 {


constexpr int kGemmRows = 128;
constexpr int kGemmKb = 64;
constexpr int kGemmThreads = 512;  // 16 warps: roles below
constexpr int kGemmProducerWarps = 8;
constexpr int kGemmMmaWarp = 8, kGemmLoadWarp = 9, kGemmEpiWarp0 = 12;
constexpr int kGemmTokTile = 256;  // tokens per work item (the MMA's largest N)
constexpr int kGemmMaxTokens = 4096;
constexpr int kGemmMaxKb = 16;  // K blocks per work item
constexpr uint32_t kErrGemmWait = 8;
// The workspace starts with a fixed header (kGemmMaxTiles words, then the
// error word), then the split partials; GEMMs of different shapes share one
// workspace.
constexpr int kGemmMaxTiles = 4096;
constexpr size_t kGemmCounterBytes = size_t(kGemmMaxTiles) * 4 + 256;

__host__ __device__ inline int gemm_np(int T) { return ((T + 15) / 16) * 16; }
inline int gemm_ttiles(int T) { return (T + kGemmTokTile - 1) / kGemmTokTile; }
__host__ __device__ inline size_t gemm_a_bytes() { return size_t(kGemmRows) * kGemmKb * 2; }
__host__ __device__ inline size_t gemm_b_bytes(int Np) { return size_t(Np) * kGemmKb * 2; }
constexpr size_t kGemmCodeStage = size_t(kGemmRows) * 32;  // 128 rows x 8 words
struct GemmLayout {
  size_t a, b, codes, scl, bia, bar, total;
};
// Ring of `S` stages (A tile, B tile, the block's codes), then per item slot
// (2) the tile's scales and biases, then the barriers.
__host__ __device__ inline GemmLayout gemm_layout(int Np, int S, int K) {
  GemmLayout L;
  L.a = 0;
  L.b = L.a + size_t(S) * gemm_a_bytes();
  L.codes = L.b + size_t(S) * gemm_b_bytes(Np);
  L.scl = L.codes + size_t(S) * kGemmCodeStage;
  L.bia = L.scl + 2 * size_t(kGemmRows) * (K / 64) * 2;
  L.bar = (L.bia + 2 * size_t(kGemmRows) * (K / 64) * 2 + 15) & ~size_t(15);
  L.total = L.bar + 256;
  return L;
}
__host__ __device__ inline uint32_t gemm_tmem_cols(int Np) {
  uint32_t c = 32;
  while (c < uint32_t(2 * Np)) c <<= 1;  // two accumulators
  return c;
}

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

Q35_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Warp roles (persistent CTA over work items blockIdx.x, + gridDim.x, ...):
//   warps 0-7   producers: dequantise A of each K block into the ring
//   warp 8      lane 0 issues the MMAs (two TMEM accumulators, by item parity)
//   warp 9      lane 0 stages: per item the tile's scales/biases (bulk copy),
//               per K block the codes and the activations (2-D TMA)
//   warps 12-15 epilogue: TMEM -> outputs (or split partials + reduction)
// Barriers: lfull[s] (loads landed), full[s] (A written, 8 producer warps),
// empty[s] (MMAs of the stage done, tcgen05.commit), wfull/wempty[w] (item
// scales), afull/aempty[a] (accumulator ready / drained). Every wait is
// bounded; after a failure the roles leave their loops.
__global__ void __launch_bounds__(kGemmThreads, 1) k_qgemm(const __grid_constant__ QGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, KG = K / 64, nkb = K / kGemmKb;
  const int T = a.T, Np = a.Np, S = a.stages;
  const int tiles = a.tiles, splits = a.splits, ttiles = a.ttiles, nitems = tiles * ttiles * splits;
  const GemmLayout L = gemm_layout(Np, S, K);
  uint8_t* As = smem + L.a;
  uint8_t* Bs = smem + L.b;
  uint8_t* Cs = smem + L.codes;
  uint16_t* scl = reinterpret_cast<uint16_t*>(smem + L.scl);
  uint16_t* bia = reinterpret_cast<uint16_t*>(smem + L.bia);
  uint64_t* lfull = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* full = lfull + 4;
  uint64_t* empty = full + 4;
  uint64_t* wfull = empty + 4;
  uint64_t* wempty = wfull + 2;
  uint64_t* afull = wempty + 2;
  uint64_t* aempty = afull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(aempty + 2);
  volatile int* bad = reinterpret_cast<volatile int*>(tslot + 1);
  const uint32_t cols = gemm_tmem_cols(Np);
  const size_t sgs = size_t(kGemmRows) * KG;  // scale/bias slot stride (elements)

  if (warp == 0) tc_alloc(tslot, cols);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&lfull[s], 1);
      mbar_init(&full[s], kGemmProducerWarps);
      mbar_init(&empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&wfull[w], 1);
      mbar_init(&wempty[w], kGemmProducerWarps);
      mbar_init(&afull[w], 1);
      mbar_init(&aempty[w], 4);
    }
    fence_mbar_init();
    // the swizzled operand tiles need 1024-byte aligned bases
    *bad = (smem_u32(smem) & 1023u) != 0u;
    if (*bad && a.err) atomicCAS(a.err, 0u, kErrGemmWait);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch();  // dependents may start staging their constants
  // everything but the loader's first scale copies and the producers (shared
  // memory only) follows the previous kernel
  if (warp == kGemmMmaWarp || warp >= kGemmEpiWarp0) pdl_wait();
  auto wait = [&](uint64_t* b, uint32_t parity) {
    if (*bad) return false;
    if (!mbar_wait_limit(b, parity, kWaitLimit, a.err, kErrGemmWait)) {
      *bad = 1;
      return false;
    }
    return true;
  };
  // item = (row tile, token tile, split), splits innermost and then the token
  // tiles, so CTAs running side by side share a weight tile in L2
  auto item_geom = [&](int item, int& tile, int& sp, int& seg, int& row0, int& nrows, int& grow0, int& kb0,
                       int& nit, int& tt) {
    sp = item % splits;
    const int rest = item / splits;
    tt = rest % ttiles;
    tile = rest / ttiles;
    int stile0;
    seg = gemm_seg_of(a, tile, &stile0, &grow0);
    row0 = (tile - stile0) * kGemmRows;
    nrows = min(kGemmRows, a.seg[seg].rows - row0);
    kb0 = sp * a.kblocks;
    nit = min(nkb, kb0 + a.kblocks) - kb0;
  };

  if (warp == kGemmLoadWarp && lane == 0) {
    // ---------------- loader ----------------
    // scales are constants: the first item's may load before the dependency wait
    int g = 0;
    for (int item = blockIdx.x, j = 0; item < nitems && !*bad; item += gridDim.x, ++j) {
      int tile, sp, seg, row0, nrows, grow0, kb0, nit, tt;
      item_geom(item, tile, sp, seg, row0, nrows, grow0, kb0, nit, tt);
      const int w = j & 1;
      if (j >= 2 && !wait(&wempty[w], uint32_t((j >> 1) - 1) & 1u)) break;
      const uint32_t sb = uint32_t(nrows) * KG * 2;
      mbar_expect_tx(&wfull[w], 2 * sb);
      bulk_g2s(scl + w * sgs, a.seg[seg].s + size_t(row0) * KG, sb, &wfull[w]);
      bulk_g2s(bia + w * sgs, a.seg[seg].b + size_t(row0) * KG, sb, &wfull[w]);
      if (j == 0) pdl_wait();  // the activations come from the previous kernel
      for (int it = 0; it < nit; ++it, ++g) {
        const int s = g % S, u = g / S;
        if (u >= 1 && !wait(&empty[s], uint32_t(u - 1) & 1u)) break;
        mbar_expect_tx(&lfull[s], uint32_t(kGemmCodeStage + gemm_b_bytes(Np)));
        tma_load_2d(Cs + s * kGemmCodeStage, &a.cmap[seg], (kb0 + it) * 8, row0, &lfull[s]);
        tma_load_2d(Bs + s * gemm_b_bytes(Np), &a.xmap, (kb0 + it) * kGemmKb, tt * Np, &lfull[s]);
      }
    }
  } else if (warp < kGemmProducerWarps) {
    // ---------------- producers ----------------
    const int r = tid & (kGemmRows - 1), half = tid >> 7;
    int g = 0;
    for (int item = blockIdx.x, j = 0; item < nitems && !*bad; item += gridDim.x, ++j) {
      int tile, sp, seg, row0, nrows, grow0, kb0, nit, tt;
      item_geom(item, tile, sp, seg, row0, nrows, grow0, kb0, nit, tt);
      const int w = j & 1;
      if (!wait(&wfull[w], uint32_t(j >> 1) & 1u)) break;
      const bool rok = r < nrows;
      for (int it = 0; it < nit; ++it, ++g) {
        const int s = g % S, u = g / S, kb = kb0 + it;
        if (!wait(&lfull[s], uint32_t(u) & 1u)) break;
        const uint4 c = *reinterpret_cast<const uint4*>(Cs + s * kGemmCodeStage + r * 32 + half * 16);
        const float sc = rok ? bf2f(scl[w * sgs + size_t(r) * KG + kb]) : 0.0f;
        const float bi = rok ? bf2f(bia[w * sgs + size_t(r) * KG + kb]) : 0.0f;
        const uint32_t words[4] = {c.x, c.y, c.z, c.w};
        // packed bf16: the nibbles at word positions (e, e + 4) become the pair
        // (128 + n_e, 128 + n_{e+4}) by one LOP3 with the bf16 bits of 128; an
        // exact subtraction of 128 and one fma rounding to nearest even give
        // bf16(s q + b) (s q is exact, so this is the correctly rounded value),
        // and byte permutes restore the order (0,1) (2,3) (4,5) (6,7)
        const __nv_bfloat162 s2 = __floats2bfloat162_rn(sc, sc), b2 = __floats2bfloat162_rn(bi, bi);
        const __nv_bfloat162 m128 = __floats2bfloat162_rn(128.0f, 128.0f);
        uint8_t* A = As + s * gemm_a_bytes();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t m = ((words[q] >> (4 * e)) & 0x000f000fu) | 0x43004300u;
            const __nv_bfloat162 q2 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&m), m128);
            const __nv_bfloat162 w2 = __hfma2(s2, q2, b2);
            v[e] = *reinterpret_cast<const uint32_t*>(&w2);
          }
          const uint4 o = rok ? make_uint4(__byte_perm(v[0], v[1], 0x5410), __byte_perm(v[2], v[3], 0x5410),
                                           __byte_perm(v[0], v[1], 0x7632), __byte_perm(v[2], v[3], 0x7632))
                              : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(A + sw128_off(r, half * 4 + q)) = o;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[w]);
    }
  } else if (warp == kGemmMmaWarp && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = tc_idesc_bf16(kGemmRows, Np);
    int g = 0;
    for (int item = blockIdx.x, j = 0; item < nitems && !*bad; item += gridDim.x, ++j) {
      int tile, sp, seg, row0, nrows, grow0, kb0, nit, tt;
      item_geom(item, tile, sp, seg, row0, nrows, grow0, kb0, nit, tt);
      const int acc = j & 1;
      if (j >= 2 && !wait(&aempty[acc], uint32_t((j >> 1) - 1) & 1u)) break;
      tc_fence_after();
      const uint32_t d = tmem + uint32_t(acc * Np);
      for (int it = 0; it < nit; ++it, ++g) {
        const int s = g % S, u = g / S;
        if (!wait(&full[s], uint32_t(u) & 1u)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(As + s * gemm_a_bytes()), b0 = smem_u32(Bs + s * gemm_b_bytes(Np));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(d, tc_desc_sw128(a0 + 32 * kk, 1024), tc_desc_sw128(b0 + 32 * kk, 1024), idesc,
                      (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      tc_commit(&afull[acc]);
    }
  } else if (warp >= kGemmEpiWarp0) {
    // ---------------- epilogue ----------------
    const int e = tid - kGemmEpiWarp0 * 32;  // 0..127 = TMEM lane = tile row
    const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
    for (int item = blockIdx.x, j = 0; item < nitems && !*bad; item += gridDim.x, ++j) {
      int tile, sp, seg, row0, nrows, grow0, kb0, nit, tt;
      item_geom(item, tile, sp, seg, row0, nrows, grow0, kb0, nit, tt);
      const int acc = j & 1;
      if (!wait(&afull[acc], uint32_t(j >> 1) & 1u)) break;
      tc_fence_after();
      const QGemmSeg& sg = a.seg[seg];
      const bool rok = e < nrows;
      const int row = row0 + e, grow = grow0 + row;
      const bool splitk = splits > 1;
      const int tb = tt * Np, tn = min(Np, T - tb);
      for (int c0 = 0; c0 < tn; c0 += 8) {
        float v[8];
        tc_ld8(tmem + lane_base + uint32_t(acc * Np + c0), v);
        if (!rok) continue;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (c0 + q >= tn) break;
          const int t = tb + c0 + q;
          if (splitk) {
            a.part[(size_t(sp) * T + t) * a.rows_total + grow] = v[q];
          } else {
            uint16_t* y = sg.y + size_t(t) * sg.ystride + row;
            if (sg.res)
              *y = f2bf(__fadd_rn(bf2f(sg.res[size_t(t) * sg.ystride + row]), bfr(v[q])));
            else
              *y = f2bf(v[q]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(&aempty[acc]);
    }
  }
  __syncwarp();  // the loader and MMA lanes rejoin their warps before the barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tc_dealloc(tmem, cols);
}

// Split K: y = bf16(sum over splits in split order) (+ residual), thread =
// (row of the concatenated row space, block of 8 tokens), consecutive threads
// on consecutive rows.
__global__ void __launch_bounds__(256) k_qgemm_reduce(const __grid_constant__ QGemmArgs a) {
  pdl_wait();
  pdl_launch();
  const int R = a.rows_total, T = a.T;
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= R * ((T + 7) / 8)) return;
  const int grow = i % R, t0 = (i / R) * 8;
  int seg = 0, r0 = 0;
  while (seg + 1 < a.nseg && grow >= r0 + a.seg[seg].rows) r0 += a.seg[seg++].rows;
  const QGemmSeg& sg = a.seg[seg];
  const int row = grow - r0;
  float s8[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) s8[q] = 0.0f;
  for (int p = 0; p < a.splits; ++p) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (t0 + q < T) s8[q] = __fadd_rn(s8[q], __ldcg(&a.part[(size_t(p) * T + t0 + q) * R + grow]));
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int t = t0 + q;
    if (t >= T) break;
    uint16_t* y = sg.y + size_t(t) * sg.ystride + row;
    if (sg.res)
      *y = f2bf(__fadd_rn(bf2f(sg.res[size_t(t) * sg.ystride + row]), bfr(s8[q])));
    else
      *y = f2bf(s8[q]);
  }
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
  qgemm_plan(tiles * gemm_ttiles(a.T), a.K, &splits, &kb);
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

constexpr size_t kGemmSmemMax = 220 * 1024;  // + the 1 KB of static shared memory

cudaError_t qgemm_init() {
  return cudaFuncSetAttribute(k_qgemm, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmSmemMax));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point.
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool tmap_2d(CUtensorMap* m, CUtensorMapDataType ty, const void* base, uint64_t d0, uint64_t d1,
                    uint64_t pitch, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  auto fn = tmap_encode();
  if (!fn) return false;
  const cuuint64_t dims[2] = {d0, d1}, strides[1] = {pitch};
  const cuuint32_t box[2] = {b0, b1}, estr[2] = {1, 1};
  return fn(m, ty, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tmap_3d(CUtensorMap* m, CUtensorMapDataType ty, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
             uint64_t p1, uint64_t p2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw) {
  auto fn = tmap_encode();
  if (!fn) return false;
  const cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {p1, p2};
  const cuuint32_t box[3] = {b0, b1, b2}, estr[3] = {1, 1, 1};
  return fn(m, ty, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Validates, lays out the workspace (header with the error word, partials),
// encodes the TMA descriptors and launches (plus the split reduction).
// `zero_counters` clears the header first.
size_t qgemm_err_offset() { return size_t(kGemmMaxTiles) * 4; }

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
  a.ttiles = gemm_ttiles(a.T);
  qgemm_plan(tiles * a.ttiles, a.K, &splits, &kb);
  a.tiles = tiles;
  a.splits = splits;
  a.kblocks = kb;
  a.rows_total = gemm_rows(a);
  uint8_t* w = static_cast<uint8_t*>(ws);
  a.counters = reinterpret_cast<uint32_t*>(w);
  a.part = reinterpret_cast<float*>(w + kGemmCounterBytes);
  if (!a.err) a.err = a.counters + kGemmMaxTiles;
  a.Np = gemm_np(a.T < kGemmTokTile ? a.T : kGemmTokTile);
  a.stages = 0;
  for (int S = 4; S >= 2 && !a.stages; --S)
    if (gemm_layout(a.Np, S, a.K).total <= kGemmSmemMax) a.stages = S;
  if (!a.stages) return cudaErrorInvalidValue;
  for (int i = 0; i < a.nseg; ++i)
    if (!tmap_2d(&a.cmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, a.seg[i].w, uint64_t(a.K / 8),
                 uint64_t(a.seg[i].rows), uint64_t(a.K / 2), 8, kGemmRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  if (!tmap_2d(&a.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, uint64_t(a.K), uint64_t(a.T), uint64_t(a.K) * 2,
               kGemmKb, uint32_t(a.Np), CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (zero_counters) {
    cudaError_t e = cudaMemsetAsync(a.counters, 0, kGemmCounterBytes, st);
    if (e != cudaSuccess) return e;
  }
  const int items = tiles * a.ttiles * splits;
  const int grid = items < 148 ? items : 148;
  cudaError_t e = launch_ex(k_qgemm, dim3(grid), dim3(kGemmThreads), gemm_layout(a.Np, a.stages, a.K).total, st,
                            pdl, a);
  if (e != cudaSuccess || splits == 1) return e;
  const int work = a.rows_total * ((a.T + 7) / 8);
  return launch_ex(k_qgemm_reduce, dim3((work + 255) / 256), dim3(256), 0, st, true, a);
}

}  // namespace q35
