// Device-side helpers shared by every q35 kernel (sm_100a only).
//
// bf16 values are carried as raw uint16_t. Rounding f32 -> bf16 is
// round-to-nearest-even (the reference's `bfloat(x)` conversion). Where a
// BF16 boundary must match the CPU oracle bit-for-bit, products and sums use
// the explicitly rounded __fmul_rn/__fadd_rn forms so that the compiler
// cannot contract them into FMAs, and transcendentals are evaluated in double
// and rounded once to f32.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q35_types.h"

#define Q35_DEV __device__ __forceinline__

namespace q35 {

Q35_DEV float bf2f(uint32_t h) { return __uint_as_float(h << 16); }
Q35_DEV uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
Q35_DEV float bfr(float f) { return bf2f(f2bf(f)); }
// two floats -> two bf16 (RNE) in one word, lo first
Q35_DEV uint32_t pack_bf2(float lo, float hi) { return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16); }
Q35_DEV float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
Q35_DEV float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// round(a * b) per component, as a packed fused multiply-add with a -0
// addend (a * b + (-0) is a * b exactly, signed zeros included). The caller
// passes the -0 from a kernel parameter: with a literal -0 ptxas turns the
// instruction back into a multiply and fuses that into the add consuming it
// (measured), which it cannot do for an addend it does not know.
Q35_DEV float2 prod2(float2 a, float2 b, float2 nz) { return __ffma2_rn(a, b, nz); }

Q35_DEV float dexpf(float x) { return (float)exp((double)x); }
Q35_DEV float dlogf(float x) { return (float)log((double)x); }
Q35_DEV float drsqrtf(float x) { return (float)(1.0 / sqrt((double)x)); }

// exp for the reference's fast::exp sites (attention softmax, log-sum-exp):
// Cody-Waite reduction x = n*ln2 + r with ln2 split into a 16-bit-exact head
// and a tail, e^r from its degree-7 Taylor polynomial (|r| <= ln2/2, remainder
// below 6e-9 relative) evaluated with fmaf, and 2^n from exponent bits. Only
// IEEE-exact operations are used, so the CPU oracle computes the same bits.
Q35_DEV float fexp(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541016f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.4426950408889634f));
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.428606765330187e-06f, r);
  float p = 1.0f / 5040.0f;
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = int(n);
  if (ni >= -125) return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 126) << 23)), 2.0f);
  return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 127 + 64) << 23)), __int_as_float((127 - 64) << 23));
}

// gdn.metal:10-15 — sigmoid with a BF16 boundary after exp, add, reciprocal
// and the positive-branch subtraction.
Q35_DEV float sigmoid_bf(float x) {
  float e = bfr(dexpf(fabsf(x)));
  float d = bfr(__fadd_rn(1.0f, e));
  float y = bfr(__fdiv_rn(1.0f, d));
  return bfr(x < 0.0f ? y : __fsub_rn(1.0f, y));
}
// gdn.metal:19-23 — MLX's log1p restricted to [0,1].
Q35_DEV float log1p_mlx(float x) {
  float xp1 = __fadd_rn(1.0f, x);
  if (xp1 == 1.0f) return x;
  return __fmul_rn(x, __fdiv_rn(dlogf(xp1), __fsub_rn(xp1, 1.0f)));
}
// gdn.metal:25-29
Q35_DEV float softplus_bf(float x) {
  float e = bfr(dexpf(-fabsf(x)));
  float l = bfr(log1p_mlx(e));
  return bfr(__fadd_rn(fmaxf(x, 0.0f), l));
}
// linear_norm.metal:95-103 — SwiGLU with BF16 steps.
Q35_DEV uint16_t swiglu_bf(float g, float up) {
  float e = bfr(dexpf(fabsf(g)));
  float denom = bfr(__fadd_rn(1.0f, e));
  float prob = bfr(__fdiv_rn(1.0f, denom));
  float s = bfr(g < 0.0f ? prob : __fsub_rn(1.0f, prob));
  float silu = bfr(__fmul_rn(g, s));
  return f2bf(__fmul_rn(silu, up));
}

// xor-butterfly warp sum; every lane ends with the same value.
Q35_DEV float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
Q35_DEV float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// ---- programmatic dependent launch --------------------------------------
// Every kernel of a decode step is launched with programmatic stream
// serialisation. It may read only constants (weights) and data written two or
// more launches earlier before pdl_wait(); it triggers its dependents right
// after pdl_wait(), so when a kernel starts, the launch two places before it
// has completed.
// System-scope flag accesses for flags that other GPUs write or read over
// NVLink (sequence-split exchange).
Q35_DEV unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
Q35_DEV void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
Q35_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
Q35_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- bulk (1-D TMA) copies with an mbarrier ------------------------------
Q35_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

Q35_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
Q35_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
Q35_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
Q35_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// global -> shared bulk copy; dst/src 16-byte aligned, bytes a multiple of 16.
Q35_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
Q35_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
Q35_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each try_wait itself may
// suspend for a hardware-defined interval), records `site` in ctl->err and
// returns false. Callers then skip their compute and exit normally.
constexpr uint32_t kWaitLimit = 1u << 24;
Q35_DEV bool mbar_wait_limit(uint64_t* bar, uint32_t parity, uint32_t limit, uint32_t* err,
                             uint32_t site) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicCAS(err, 0u, site);
  return false;
}
Q35_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, Ctl* ctl, uint32_t site) {
  return mbar_wait_limit(bar, parity, kWaitLimit, ctl ? &ctl->err : nullptr, site);
}

Q35_DEV uint32_t ld_cg_u32(const uint32_t* p) { return __ldcg(p); }

}  // namespace q35
