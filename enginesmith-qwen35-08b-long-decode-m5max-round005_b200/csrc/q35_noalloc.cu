// Allocation-free variant of the decode-attention op.
//
// Some callers cannot call cudaMalloc: code that runs where the allocator is
// off limits (a custom allocator's own callbacks, a process whose device
// memory is carved up up-front by a serving framework that forbids further
// allocations, or a plugin host that hands out no workspace), and code that
// cannot afford an allocation's implicit synchronisation in the middle of its
// step. q35_op_attn_decode needs a caller-provided workspace; this variant
// instead uses a fixed scratch array that lives in the library's own device
// image, so it allocates nothing and takes no workspace.
//
// The scratch is one file-scope __device__ array of kScratchBytes per device.
// Every device that loads the library holds it until the process exits. Every
// call on a device shares it, and it keeps the last call's contents: the
// control block is rewritten at the start of each call (position, error flag,
// counters, RoPE table), and the chain partials are fully written by the
// attention kernel before the combine reads them. Calls whose execution
// overlaps on the GPU (two streams, or two host threads on one device) race on
// the scratch; serialise them.
//
// Set-up: the first call on a device (with that device current) looks up the
// scratch's device address with cudaGetSymbolAddress and sets the kernels'
// shared-memory limits. Make that first call before any stream capture on
// the device. The address is cached per device number for the life of the
// process, so calls after a cudaDeviceReset of that device are unsupported.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "q35.h"
#include "q35_kernels.h"
#include "q35_types.h"

namespace {

using namespace q35;

// Maximum scratch per device: 576 KiB. This call needs the control block
// (rounded up to 256 bytes: 512) plus the per-chain partials of 2 kv heads x
// 64 chains x 4 query heads (f32 [256] output + f32 (max, sum)): 528,896
// bytes at any context length; a static_assert below holds the layout to the
// maximum.
constexpr size_t kScratchBytes = 576 * 1024;

__device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

constexpr size_t kCtlBytes = (sizeof(Ctl) + 255) & ~size_t(255);
constexpr size_t kPartOBytes = size_t(kKvHeads) * kAttnChains * 4 * kHeadDim * 4;
constexpr size_t kPartMlBytes = size_t(kKvHeads) * kAttnChains * 4 * 2 * 4;
constexpr size_t kNeedBytes = kCtlBytes + kPartOBytes + kPartMlBytes;
static_assert(kNeedBytes <= kScratchBytes, "the attention op's scratch layout outgrew the static array");
static_assert(kNeedBytes == 528896, "scratch need changed: update the documented figure");

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_ptr[kMaxDevices] = {};

void put_err(char* err, size_t n, const char* msg) {
  if (err && n) std::snprintf(err, n, "%s", msg);
}

}  // namespace

namespace q35 {
unsigned char* noalloc_scratch(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_ptr[dev];
}
}  // namespace q35

extern "C" int q35_op_attn_decode_noalloc(const uint16_t* q_raw, const uint16_t* k_raw,
                                          const uint16_t* v_raw, const uint16_t* q_gain,
                                          const uint16_t* k_gain, uint16_t* kcache,
                                          uint16_t* vcache, uint32_t capacity, uint32_t pos,
                                          uint16_t* gated, char* err, size_t err_len,
                                          void* stream) {
  if (!q_raw || !k_raw || !v_raw || !q_gain || !k_gain || !kcache || !vcache || !gated) {
    put_err(err, err_len, "attn_decode_noalloc: null pointer argument");
    return Q35_EINVAL;
  }
  for (const void* p : {(const void*)q_raw, (const void*)k_raw, (const void*)v_raw, (const void*)q_gain,
                        (const void*)k_gain, (const void*)kcache, (const void*)vcache})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) {
      put_err(err, err_len, "attn_decode_noalloc: inputs and caches must be 16-byte aligned");
      return Q35_EINVAL;
    }
  if (capacity == 0 || capacity % kAttnChains != 0) {
    put_err(err, err_len, "attn_decode_noalloc: capacity must be a positive multiple of 64");
    return Q35_EINVAL;
  }
  if (pos >= capacity) {
    put_err(err, err_len, "attn_decode_noalloc: pos must be below capacity");
    return Q35_EINVAL;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    put_err(err, err_len, "attn_decode_noalloc: no usable current device");
    return Q35_ECUDA;
  }
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_attn_scratch);
      if (e != cudaSuccess) {
        char m[200];
        std::snprintf(m, sizeof(m), "attn_decode_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(e));
        put_err(err, err_len, m);
        return Q35_ECUDA;
      }
      e = kernels_init();
      if (e != cudaSuccess) {
        put_err(err, err_len, "attn_decode_noalloc: kernel set-up failed");
        return Q35_ECUDA;
      }
      g_ptr[dev] = static_cast<unsigned char*>(p);
    }
    base = g_ptr[dev];
  }
  cudaStream_t st = (cudaStream_t)stream;
  Ctl* ctl = reinterpret_cast<Ctl*>(base);
  float* po = reinterpret_cast<float*>(base + kCtlBytes);
  float* pml = reinterpret_cast<float*>(base + kCtlBytes + kPartOBytes);
  e = launch_ctl_position(ctl, pos, st);
  AttnArgs at = {};
  at.q_raw = q_raw;
  at.k_raw = k_raw;
  at.v_raw = v_raw;
  at.q_gain = q_gain;
  at.k_gain = k_gain;
  at.kcache = kcache;
  at.vcache = vcache;
  at.capacity = capacity;
  at.part_o = po;
  at.part_ml = pml;
  at.gated = gated;
  at.ctl = ctl;
  if (e == cudaSuccess) e = launch_attn(at, st, false);
  if (e != cudaSuccess) {
    char m[200];
    std::snprintf(m, sizeof(m), "attn_decode_noalloc: launch failed: %s", cudaGetErrorString(e));
    put_err(err, err_len, m);
    return Q35_ECUDA;
  }
  return Q35_OK;
}
