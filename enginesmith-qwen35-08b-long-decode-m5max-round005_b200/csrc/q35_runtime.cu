// q35 runtime: model loading, decode sessions (CUDA-graph token loop) and the
// op-level C ABI. Mirrors the reference host (source/src/model.rs,
// source/src/weights.rs) with CUDA streams/graphs in place of Metal command
// buffers.
#include <dirent.h>
#include <limits.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "q35.h"
#include "q35_json.h"
#include "q35_kernels.h"

using namespace q35;

namespace {

// ---------------------------------------------------------------------------
// weights (weights.rs:8-53)
// ---------------------------------------------------------------------------
struct Lin {
  const uint32_t* w = nullptr;
  const uint16_t* s = nullptr;
  const uint16_t* b = nullptr;
  int n = 0, k = 0;
};
struct LayerW {
  bool attn = false;
  const uint16_t* in_norm = nullptr;
  const uint16_t* post_norm = nullptr;
  Lin gate, up, down;
  Lin qkv, z, a, bproj, out;  // GDN
  const uint16_t *conv = nullptr, *gnorm = nullptr, *dt = nullptr;
  const float* alog = nullptr;
  Lin q, k, v, o;  // attention
  const uint16_t *qnorm = nullptr, *knorm = nullptr;
};
struct ModelW {
  uint8_t* arena = nullptr;
  size_t bytes = 0;
  Lin embed;
  const uint16_t* norm = nullptr;
  LayerW L[kLayers];
};

struct TensorRec {
  int file = 0;
  std::string dtype;
  std::vector<size_t> shape;
  size_t offset = 0, bytes = 0;
  size_t dev_off = 0;
  bool used = false;
};

bool read_file(const std::string& path, std::vector<char>& out, std::string& err) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    err = "cannot open " + path;
    return false;
  }
  std::fseek(f, 0, SEEK_END);
  long n = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  out.resize(size_t(n));
  size_t got = n > 0 ? std::fread(out.data(), 1, size_t(n), f) : 0;
  std::fclose(f);
  if (got != size_t(n)) {
    err = "short read " + path;
    return false;
  }
  return true;
}

class Loader {
 public:
  std::string err;
  bool open(const std::string& dir) {
    std::vector<char> cfg;
    if (!read_file(dir + "/config.json", cfg, err)) return false;
    q35json::Value cv;
    if (!q35json::parse(std::string(cfg.begin(), cfg.end()), cv, err)) return false;
    const q35json::Value* tc = cv.get("text_config");
    uint64_t hs = 0, nl = 0, vs = 0;
    if (!tc || !tc->get("hidden_size") || !tc->get("hidden_size")->as_u64(hs) ||
        !tc->get("num_hidden_layers") || !tc->get("num_hidden_layers")->as_u64(nl) ||
        !tc->get("vocab_size") || !tc->get("vocab_size")->as_u64(vs) || hs != 1024 || nl != 24 ||
        vs != 248320) {
      err = "unsupported model configuration";  // weights.rs:14-15
      return false;
    }
    DIR* d = opendir(dir.c_str());
    if (!d) {
      err = "cannot list " + dir;
      return false;
    }
    while (dirent* e = readdir(d)) {
      std::string n = e->d_name;
      if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files_.push_back(dir + "/" + n);
    }
    closedir(d);
    std::sort(files_.begin(), files_.end());
    if (files_.empty()) {
      err = "no safetensors weights";
      return false;
    }
    data_.resize(files_.size());
    for (size_t fi = 0; fi < files_.size(); ++fi) {
      std::vector<char>& bytes = data_[fi];
      if (!read_file(files_[fi], bytes, err)) return false;
      if (bytes.size() < 8) {
        err = "short safetensors file";
        return false;
      }
      uint64_t hn = 0;
      std::memcpy(&hn, bytes.data(), 8);
      if (hn > bytes.size() - 8) {
        err = "invalid safetensors header";
        return false;
      }
      q35json::Value h;
      if (!q35json::parse(std::string(bytes.data() + 8, size_t(hn)), h, err)) return false;
      if (h.type != q35json::Value::Object) {
        err = "invalid header";
        return false;
      }
      const size_t data_len = bytes.size() - 8 - size_t(hn);
      for (auto& kv : h.obj) {
        const std::string& name = kv.first;
        if (name == "__metadata__") continue;
        static const std::string pre = "language_model.model.";
        if (name.compare(0, pre.size(), pre) != 0) continue;
        TensorRec t;
        t.file = int(fi);
        const q35json::Value* dt = kv.second.get("dtype");
        const q35json::Value* sh = kv.second.get("shape");
        const q35json::Value* of = kv.second.get("data_offsets");
        if (!dt || dt->type != q35json::Value::String) {
          err = "missing dtype";
          return false;
        }
        t.dtype = dt->str;
        size_t elem = 0;
        if (t.dtype == "U32" || t.dtype == "F32") elem = 4;
        else if (t.dtype == "BF16") elem = 2;
        else {
          err = "unsupported dtype " + t.dtype;
          return false;
        }
        if (!sh || sh->type != q35json::Value::Array) {
          err = "missing shape";
          return false;
        }
        size_t count = 1;
        for (auto& x : sh->arr) {
          uint64_t v;
          if (!x.as_u64(v)) {
            err = "invalid shape";
            return false;
          }
          t.shape.push_back(size_t(v));
          count *= size_t(v);
        }
        uint64_t a = 0, b = 0;
        if (!of || of->type != q35json::Value::Array || of->arr.size() != 2 || !of->arr[0].as_u64(a) ||
            !of->arr[1].as_u64(b)) {
          err = "invalid offset";
          return false;
        }
        if (b < a || b > data_len || b - a != count * elem) {
          err = "tensor bounds: " + name;
          return false;
        }
        t.offset = 8 + size_t(hn) + size_t(a);
        t.bytes = size_t(b - a);
        std::string key = name.substr(pre.size());
        for (auto& r : recs_)
          if (r.first == key) {
            err = "duplicate tensor " + key;
            return false;
          }
        recs_.emplace_back(key, t);
      }
    }
    if (recs_.size() != 694) {
      err = "expected 694 text tensors, got " + std::to_string(recs_.size());
      return false;
    }
    return true;
  }
  // Upload every tensor to one device arena, each 256-byte aligned (the bulk
  // copies need 16-byte aligned sources; safetensors offsets are not).
  bool upload(ModelW& M) {
    size_t total = 0;
    for (auto& r : recs_) {
      r.second.dev_off = total;
      total += (r.second.bytes + 255) & ~size_t(255);
    }
    if (cudaMalloc(&M.arena, total) != cudaSuccess) {
      err = "cudaMalloc of " + std::to_string(total) + " weight bytes failed";
      return false;
    }
    M.bytes = total;
    for (auto& r : recs_) {
      const TensorRec& t = r.second;
      if (cudaMemcpy(M.arena + t.dev_off, data_[size_t(t.file)].data() + t.offset, t.bytes,
                     cudaMemcpyHostToDevice) != cudaSuccess) {
        err = "weight upload failed";
        return false;
      }
    }
    arena_ = M.arena;
    data_.clear();
    data_.shrink_to_fit();
    return true;
  }
  // Weights::take (weights.rs:45-49)
  const void* take(const std::string& name, std::initializer_list<size_t> shape, const char* dtype) {
    for (auto& r : recs_)
      if (r.first == name) {
        TensorRec& t = r.second;
        if (t.used || t.dtype != dtype || t.shape != std::vector<size_t>(shape)) {
          if (err.empty()) err = "wrong shape/dtype for " + name;
          return nullptr;
        }
        t.used = true;
        return arena_ + t.dev_off;
      }
    if (err.empty()) err = "missing " + name;
    return nullptr;
  }
  // Weights::linear (weights.rs:50-52)
  Lin linear(const std::string& name, int n, int k) {
    Lin l;
    l.w = (const uint32_t*)take(name + ".weight", {size_t(n), size_t(k / 8)}, "U32");
    l.s = (const uint16_t*)take(name + ".scales", {size_t(n), size_t(k / 64)}, "BF16");
    l.b = (const uint16_t*)take(name + ".biases", {size_t(n), size_t(k / 64)}, "BF16");
    l.n = n;
    l.k = k;
    return l;
  }
  // Weights::done (weights.rs:53)
  bool done() {
    if (!err.empty()) return false;
    for (auto& r : recs_)
      if (!r.second.used) {
        err = "unused text weights: " + r.first;
        return false;
      }
    return true;
  }

 private:
  std::vector<std::string> files_;
  std::vector<std::vector<char>> data_;
  std::vector<std::pair<std::string, TensorRec>> recs_;
  uint8_t* arena_ = nullptr;
};

// model.rs:41-78
bool bind_model(Loader& ld, ModelW& M) {
  M.embed = ld.linear("embed_tokens", kVocab, kHidden);
  M.norm = (const uint16_t*)ld.take("norm.weight", {1024}, "BF16");
  for (int l = 0; l < kLayers; ++l) {
    LayerW& L = M.L[l];
    const std::string p = "layers." + std::to_string(l);
    L.in_norm = (const uint16_t*)ld.take(p + ".input_layernorm.weight", {1024}, "BF16");
    L.post_norm = (const uint16_t*)ld.take(p + ".post_attention_layernorm.weight", {1024}, "BF16");
    L.gate = ld.linear(p + ".mlp.gate_proj", kMlp, kHidden);
    L.up = ld.linear(p + ".mlp.up_proj", kMlp, kHidden);
    L.down = ld.linear(p + ".mlp.down_proj", kHidden, kMlp);
    L.attn = (l % 4) == 3;
    if (L.attn) {
      const std::string a = p + ".self_attn";
      L.q = ld.linear(a + ".q_proj", 4096, 1024);
      L.k = ld.linear(a + ".k_proj", 512, 1024);
      L.v = ld.linear(a + ".v_proj", 512, 1024);
      L.o = ld.linear(a + ".o_proj", 1024, 2048);
      L.qnorm = (const uint16_t*)ld.take(a + ".q_norm.weight", {256}, "BF16");
      L.knorm = (const uint16_t*)ld.take(a + ".k_norm.weight", {256}, "BF16");
    } else {
      const std::string a = p + ".linear_attn";
      L.qkv = ld.linear(a + ".in_proj_qkv", 6144, 1024);
      L.z = ld.linear(a + ".in_proj_z", 2048, 1024);
      L.a = ld.linear(a + ".in_proj_a", 16, 1024);
      L.bproj = ld.linear(a + ".in_proj_b", 16, 1024);
      L.out = ld.linear(a + ".out_proj", 1024, 2048);
      L.conv = (const uint16_t*)ld.take(a + ".conv1d.weight", {6144, 4, 1}, "BF16");
      L.gnorm = (const uint16_t*)ld.take(a + ".norm.weight", {128}, "BF16");
      L.dt = (const uint16_t*)ld.take(a + ".dt_bias", {16}, "BF16");
      L.alog = (const float*)ld.take(a + ".A_log", {16}, "F32");
    }
  }
  return ld.done();
}

std::mutex g_init_mu;
uint64_t g_init_mask = 0;
cudaError_t ensure_kernels_init() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (dev < 64 && (g_init_mask >> dev) & 1) return cudaSuccess;
  e = kernels_init();
  if (e == cudaSuccess) e = chunk_kernels_init();
  if (e == cudaSuccess) e = qgemm_init();
  if (e == cudaSuccess) e = prompt_kernels_init();
  if (e == cudaSuccess && dev < 64) g_init_mask |= uint64_t(1) << dev;
  return e;
}

// The session options q35_open accepts (host arithmetic only).
bool validate_opts(const q35_opts* o, std::string& m) {
  const uint32_t cap = o && o->capacity ? o->capacity : kDefaultCapacity;
  const uint32_t chunk = o && o->prompt_chunk ? o->prompt_chunk : uint32_t(kPromptChunk);
  if (cap % kAttnChains != 0 || cap < kAttnChains || cap > (1u << 30)) {
    m = "capacity must be a positive multiple of 64";
    return false;
  }
  if (chunk < 32 || chunk > uint32_t(kPromptChunk) || chunk % 32 != 0) {
    m = "prompt_chunk must be a multiple of 32 in 32..2048";
    return false;
  }
  if (o && (o->decode_batch > 1024 || o->prefill_batch > 1024)) {
    m = "decode_batch and prefill_batch must be at most 1024";
    return false;
  }
  return true;
}

void copy_err(char* dst, size_t n, const std::string& m) {
  if (dst && n) std::snprintf(dst, n, "%s", m.c_str());
}

}  // namespace

// ---------------------------------------------------------------------------
// session
// ---------------------------------------------------------------------------
struct q35_session {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t capacity = kDefaultCapacity;
  int dbatch = 8, pbatch = 16;
  ModelW M;
  uint8_t* buf = nullptr;  // one allocation for all scratch/state
  Ctl* ctl = nullptr;
  uint16_t *h = nullptr, *conv_out = nullptr, *z = nullptr, *ab = nullptr, *y = nullptr;
  uint16_t *q = nullptr, *k = nullptr, *v = nullptr, *gated = nullptr, *act = nullptr;
  uint16_t *logits = nullptr, *lse = nullptr;
  float *attn_po = nullptr, *attn_pml = nullptr, *head_part = nullptr;
  float* zs = nullptr;  // z * sigmoid(z) of the step's GDN layer [2048]
  uint32_t *seq = nullptr, *out_tokens = nullptr;
  float* state = nullptr;
  uint16_t* hist = nullptr;
  uint16_t* kv = nullptr;  // [6 layers][K|V][2][capacity][256]
  cudaGraphExec_t gdec1 = nullptr, gdecN = nullptr, gpre1 = nullptr, gpreN = nullptr;
  // kernel launches in one replay of the decode graphs (counted at capture)
  uint32_t kn_dec1 = 0, kn_decN = 0;
  uint64_t launches = 0;  // decode-graph kernel launches since the last q35_launch_count reset
  // in-flight window of the token loop: the host waits on the event of the
  // launch kInflight places back before it queues the next one
  cudaEvent_t inflight[kInflight] = {};
  // prompt chunks of kPrefillTokens tokens (per-token rows of each buffer)
  bool chunked = true;
  cudaGraphExec_t gchunk = nullptr;
  uint16_t *c_h = nullptr, *c_conv = nullptr, *c_z = nullptr, *c_ab = nullptr, *c_y = nullptr;
  uint16_t *c_q = nullptr, *c_k = nullptr, *c_v = nullptr, *c_gated = nullptr, *c_act = nullptr;
  float* c_rope = nullptr;
  float* c_zs = nullptr;  // z * sigmoid(z) of the chunk's tokens [16][2048]
  // prompts on the tensor cores (Q35_FLAG_TENSOR_PROMPT): chunks of up to
  // prompt_chunk tokens; buffers allocated on first use
  bool tensor_prompt = false;
  int prompt_chunk = kPromptChunk;
  uint8_t* pbuf = nullptr;
  uint16_t *p_h = nullptr, *p_xn = nullptr, *p_raw = nullptr, *p_z = nullptr, *p_ab = nullptr, *p_conv = nullptr;
  uint16_t *p_y = nullptr, *p_gated = nullptr, *p_q = nullptr, *p_k = nullptr, *p_v = nullptr, *p_gu = nullptr;
  uint16_t *p_act = nullptr, *p_qn = nullptr;
  float *p_zs = nullptr, *p_rope = nullptr, *p_kq = nullptr, *p_gb = nullptr, *p_vv = nullptr;
  float *p_opart = nullptr, *p_oml = nullptr, *p_omax = nullptr;
  uint8_t* p_gws = nullptr;
  size_t p_gws_bytes = 0;
  uint32_t position = 0;
  bool has_pending = false;
  uint32_t pending = 0;
  std::atomic<bool> cancelled{false};
  std::string err;
  std::string model_id;  // canonical model directory (batched sessions must share it)
  uint32_t epoch = 0;    // reset generation, tags the sequence-split exchange
  // sequence split (xworld > 1 once connected): this rank's exchange buffers
  // (records, then flags), the peers' mapped buffers and the device tables
  int xrank = 0, xworld = 1, xpend_world = 0;
  uint32_t xwait_ms = 0;  // bound of the exchange wait (0: the kernel's 10 s)
  uint8_t* xbuf = nullptr;
  uint16_t* xkv = nullptr;  // one layer's K/V at full capacity: the tensor-core prompt's rows before the split keeps its share
  std::vector<void*> xpeer;
  void** xtab = nullptr;  // [xworld] record pointers, then [xworld] flag pointers

  // K/V capacity of this rank's caches (the local share under a sequence split)
  uint32_t kv_capacity() const {
    if (xworld <= 1) return capacity;
    const uint32_t per = (capacity + uint32_t(xworld) - 1) / uint32_t(xworld);
    return (per + kAttnChains - 1) / kAttnChains * kAttnChains;
  }
  uint16_t* kcache(int ai) { return kv + size_t(ai) * 2 * kKvHeads * capacity * kHeadDim; }
  uint16_t* vcache(int ai) { return kcache(ai) + size_t(kKvHeads) * capacity * kHeadDim; }
};

namespace {

int set_err(q35_session* s, int code, const std::string& m) {
  if (s) s->err = m;
  return code;
}

// Attention-launch fields of the session's sequence split (none when off).
void split_attn_args(const q35_session* s, AttnArgs& at, int ai) {
  at.capacity = s->kv_capacity();
  if (s->xworld <= 1) return;
  at.xrank = s->xrank;
  at.xworld = s->xworld;
  at.xlayer = ai;
  at.xwait_ms = s->xwait_ms;
  at.xrecv = reinterpret_cast<float* const*>(s->xtab);
  at.xflag = reinterpret_cast<unsigned long long* const*>(s->xtab + s->xworld);
}

// One decode step: model.rs:228-307 for rows == 1 (+ the head when `head`).
cudaError_t enqueue_step(q35_session* s, bool head, bool first) {
  const ModelW& M = s->M;
  cudaStream_t st = s->stream;
  bool pdl = !first;
  cudaError_t e = cudaSuccess;
#define Q35_L(x)               \
  do {                         \
    e = (x);                   \
    if (e != cudaSuccess) return e; \
    pdl = true;                \
  } while (0)
  int gi = 0, ai = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerW& L = M.L[l];
    if (!L.attn) {
      QmvArgs a = {};
      a.seg[0] = {L.qkv.w, L.qkv.s, L.qkv.b, nullptr, 6144};
      a.seg[1] = {L.z.w, L.z.s, L.z.b, s->z, 2048};
      a.seg[2] = {L.a.w, L.a.s, L.a.b, s->ab, 16};
      a.seg[3] = {L.bproj.w, L.bproj.s, L.bproj.b, s->ab + 16, 16};
      a.nseg = 4;
      a.K = 1024;
      a.units = 8224;
      a.units_per_cta = 56;
      a.pro = l == 0 ? kProEmbedRms : kProRms;
      a.epi = kEpiGdnConv;
      a.x = s->h;
      a.gain = L.in_norm;
      a.h_out = s->h;
      a.ew = M.embed.w;
      a.es = M.embed.s;
      a.eb = M.embed.b;
      a.seq = s->seq;
      a.hist = s->hist + size_t(gi) * 3 * kGdnConv;
      a.convw = L.conv;
      a.conv_out = s->conv_out;
      a.zs_out = s->zs;
      a.ctl = s->ctl;
      Q35_L(launch_qmv(a, st, pdl));
      RecurArgs r = {};
      r.conv = s->conv_out;
      r.a_raw = s->ab;
      r.b_raw = s->ab + 16;
      r.a_log = L.alog;
      r.dt_bias = L.dt;
      r.state = s->state + size_t(gi) * kGdnHeads * 128 * 128;
      r.y = s->y;
      r.ctl = s->ctl;
      r.advance_pos = l == 0;
      Q35_L(launch_recur(r, st, pdl));
      QmvArgs o = {};
      o.seg[0] = {L.out.w, L.out.s, L.out.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProNormGate;
      o.gy = s->y;
      o.gz = s->z;
      o.gzs = s->zs;
      o.gw = L.gnorm;
      o.epi = kEpiResAdd;
      o.res = s->h;
      o.ctl = s->ctl;
      Q35_L(launch_qmv(o, st, pdl));
      ++gi;
    } else {
      QmvArgs a = {};
      a.seg[0] = {L.q.w, L.q.s, L.q.b, s->q, 4096};
      a.seg[1] = {L.k.w, L.k.s, L.k.b, s->k, 512};
      a.seg[2] = {L.v.w, L.v.s, L.v.b, s->v, 512};
      a.nseg = 3;
      a.K = 1024;
      a.units = 5120;
      a.units_per_cta = 36;
      a.pro = kProRms;
      a.x = s->h;
      a.gain = L.in_norm;
      a.epi = kEpiStore;
      a.ctl = s->ctl;
      Q35_L(launch_qmv(a, st, pdl));
      AttnArgs at = {};
      at.q_raw = s->q;
      at.k_raw = s->k;
      at.v_raw = s->v;
      at.q_gain = L.qnorm;
      at.k_gain = L.knorm;
      at.kcache = s->kcache(ai);
      at.vcache = s->vcache(ai);
      at.capacity = s->capacity;
      at.part_o = s->attn_po;
      at.part_ml = s->attn_pml;
      at.gated = s->gated;
      at.ctl = s->ctl;
      split_attn_args(s, at, ai);
      Q35_L(launch_attn(at, st, pdl));
      QmvArgs o = {};
      o.seg[0] = {L.o.w, L.o.s, L.o.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProPlain;
      o.x = s->gated;
      o.epi = kEpiResAdd;
      o.res = s->h;
      o.ctl = s->ctl;
      Q35_L(launch_qmv(o, st, pdl));
      ++ai;
    }
    QmvArgs m = {};
    m.seg[0] = {L.gate.w, L.gate.s, L.gate.b, s->act, kMlp};
    m.seg[1] = {L.up.w, L.up.s, L.up.b, nullptr, kMlp};
    m.nseg = 2;
    m.K = 1024;
    m.units = kMlp;
    m.units_per_cta = 25;
    m.pro = kProRms;
    m.x = s->h;
    m.gain = L.post_norm;
    m.epi = kEpiSwiglu;
    m.ctl = s->ctl;
    Q35_L(launch_qmv(m, st, pdl));
    QmvArgs d = {};
    d.seg[0] = {L.down.w, L.down.s, L.down.b, nullptr, 1024};
    d.nseg = 1;
    d.K = kMlp;
    d.units = 1024;
    d.units_per_cta = 7;
    d.pro = kProPlain;
    d.x = s->act;
    d.epi = kEpiResAdd;
    d.res = s->h;
    d.ctl = s->ctl;
    Q35_L(launch_qmv(d, st, pdl));
  }
  if (head) {
    HeadArgs hd = {};
    hd.w = M.embed.w;
    hd.s = M.embed.s;
    hd.b = M.embed.b;
    hd.x = s->h;
    hd.gain = M.norm;
    hd.logits = s->logits;
    hd.part = s->head_part;
    hd.seq = s->seq;
    hd.out_tokens = s->out_tokens;
    hd.seq_len = s->capacity + 1;
    hd.out_len = s->capacity;
    hd.lse_out = s->lse;
    hd.ctl = s->ctl;
    Q35_L(launch_head(hd, st, pdl));
  }
#undef Q35_L
  return e;
}

// One prompt chunk: kPrefillTokens consecutive prompt tokens through all 24
// layers (no head), with the decode step's arithmetic per token. Matvecs and
// the GDN recurrence take the whole chunk per launch; attention runs once per
// token (token t attends to keys 0..pos+t, its own key appended first).
cudaError_t enqueue_chunk(q35_session* s) {
  const ModelW& M = s->M;
  cudaStream_t st = s->stream;
  constexpr int T = kPrefillTokens;
  bool pdl = false;
  cudaError_t e = cudaSuccess;
#define Q35_C(x)                    \
  do {                              \
    e = (x);                        \
    if (e != cudaSuccess) return e; \
    pdl = true;                     \
  } while (0)
  auto chunk_args = [&](QmvArgs& a) {
    a.ntok = T;
    a.sub = chunk_sub_tokens(a);
    a.ctl = s->ctl;
  };
  int gi = 0, ai = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerW& L = M.L[l];
    if (!L.attn) {
      QmvArgs a = {};
      a.seg[0] = {L.qkv.w, L.qkv.s, L.qkv.b, nullptr, 6144};
      a.seg[1] = {L.z.w, L.z.s, L.z.b, s->c_z, 2048};
      a.seg[2] = {L.a.w, L.a.s, L.a.b, s->c_ab, 16};
      a.seg[3] = {L.bproj.w, L.bproj.s, L.bproj.b, s->c_ab + 16, 16};
      a.ystride[1] = 2048;
      a.ystride[2] = 32;
      a.ystride[3] = 32;
      a.nseg = 4;
      a.K = 1024;
      a.units = 8224;
      a.units_per_cta = 56;
      a.pro = l == 0 ? kProEmbedRms : kProRms;
      a.epi = kEpiGdnConv;
      a.x = s->c_h;
      a.gain = L.in_norm;
      a.h_out = s->c_h;
      a.ew = M.embed.w;
      a.es = M.embed.s;
      a.eb = M.embed.b;
      a.seq = s->seq;
      a.rope_out = s->c_rope;
      a.hist = s->hist + size_t(gi) * 3 * kGdnConv;
      a.convw = L.conv;
      a.conv_out = s->c_conv;
      chunk_args(a);
      Q35_C(launch_qmv_chunk(a, st, pdl));
      RecurArgs r = {};
      r.conv = s->c_conv;
      r.a_raw = s->c_ab;
      r.b_raw = s->c_ab + 16;
      r.a_log = L.alog;
      r.dt_bias = L.dt;
      r.state = s->state + size_t(gi) * kGdnHeads * 128 * 128;
      r.y = s->c_y;
      r.z = s->c_z;
      r.zs = s->c_zs;
      r.ctl = s->ctl;
      r.advance_pos = l == 0;
      r.ntok = T;
      Q35_C(launch_recur_chunk(r, st, pdl));
      QmvArgs o = {};
      o.seg[0] = {L.out.w, L.out.s, L.out.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProNormGate;
      o.gy = s->c_y;
      o.gz = s->c_z;
      o.gzs = s->c_zs;
      o.gw = L.gnorm;
      o.epi = kEpiResAdd;
      o.res = s->c_h;
      chunk_args(o);
      Q35_C(launch_qmv_chunk(o, st, pdl));
      ++gi;
    } else {
      QmvArgs a = {};
      a.seg[0] = {L.q.w, L.q.s, L.q.b, s->c_q, 4096};
      a.seg[1] = {L.k.w, L.k.s, L.k.b, s->c_k, 512};
      a.seg[2] = {L.v.w, L.v.s, L.v.b, s->c_v, 512};
      a.ystride[0] = kQProj;
      a.ystride[1] = 512;
      a.ystride[2] = 512;
      a.nseg = 3;
      a.K = 1024;
      a.units = 5120;
      a.units_per_cta = 36;
      a.pro = kProRms;
      a.x = s->c_h;
      a.gain = L.in_norm;
      a.epi = kEpiStore;
      chunk_args(a);
      Q35_C(launch_qmv_chunk(a, st, pdl));
      for (int t = 0; t < T; ++t) {
        AttnArgs at = {};
        at.q_raw = s->c_q + size_t(t) * kQProj;
        at.k_raw = s->c_k + size_t(t) * 512;
        at.v_raw = s->c_v + size_t(t) * 512;
        at.q_gain = L.qnorm;
        at.k_gain = L.knorm;
        at.kcache = s->kcache(ai);
        at.vcache = s->vcache(ai);
        at.capacity = s->capacity;
        at.part_o = s->attn_po;
        at.part_ml = s->attn_pml;
        at.gated = s->c_gated + size_t(t) * 2048;
        at.ctl = s->ctl;
        at.pos_add = t;
        at.rope = s->c_rope + 64 * t;
        split_attn_args(s, at, ai);
        Q35_C(launch_attn(at, st, pdl));
      }
      QmvArgs o = {};
      o.seg[0] = {L.o.w, L.o.s, L.o.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProPlain;
      o.x = s->c_gated;
      o.epi = kEpiResAdd;
      o.res = s->c_h;
      chunk_args(o);
      Q35_C(launch_qmv_chunk(o, st, pdl));
      ++ai;
    }
    QmvArgs m = {};
    m.seg[0] = {L.gate.w, L.gate.s, L.gate.b, s->c_act, kMlp};
    m.seg[1] = {L.up.w, L.up.s, L.up.b, nullptr, kMlp};
    m.ystride[0] = kMlp;
    m.nseg = 2;
    m.K = 1024;
    m.units = kMlp;
    m.units_per_cta = 25;
    m.pro = kProRms;
    m.x = s->c_h;
    m.gain = L.post_norm;
    m.epi = kEpiSwiglu;
    chunk_args(m);
    Q35_C(launch_qmv_chunk(m, st, pdl));
    QmvArgs d = {};
    d.seg[0] = {L.down.w, L.down.s, L.down.b, nullptr, 1024};
    d.nseg = 1;
    d.K = kMlp;
    d.units = 1024;
    d.units_per_cta = 7;
    d.pro = kProPlain;
    d.x = s->c_act;
    d.epi = kEpiResAdd;
    d.res = s->c_h;
    chunk_args(d);
    Q35_C(launch_qmv_chunk(d, st, pdl));
  }
#undef Q35_C
  return e;
}

cudaError_t capture_chunk(q35_session* s, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return e;
  const cudaError_t le = enqueue_chunk(s);
  e = cudaStreamEndCapture(s->stream, &g);
  if (le != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return le;
  }
  if (e != cudaSuccess) return e;
  e = cudaGraphInstantiate(out, g, 0);
  // upload now, so that the first replay (inside a request or a timed region)
  // does not pay for it
  if (e == cudaSuccess) e = cudaGraphUpload(*out, s->stream);
  cudaGraphDestroy(g);
  return e;
}

// Buffers of the tensor-core prompt route, sized for prompt_chunk tokens (the
// attention partials for the session's capacity); allocated on first use.
cudaError_t ensure_prompt_buffers(q35_session* s) {
  if (s->pbuf) return cudaSuccess;
  const size_t N = size_t(s->prompt_chunk);
  const size_t items = prompt_attn_items_max(s->prompt_chunk, s->capacity);
  // the largest GEMM workspace over every chunk length (a shorter last chunk
  // may split K further)
  auto ws = [&](std::initializer_list<int> rows, int K, int T) {
    QGemmArgs g = {};
    for (int r : rows) g.seg[g.nseg++].rows = r;
    g.K = K;
    g.T = T;
    return qgemm_workspace_bytes(g);
  };
  s->p_gws_bytes = 0;
  for (int T = 1; T <= int(N); ++T)
    for (size_t w : {ws({kGdnConv, 2048, 16, 16}, kHidden, T), ws({kHidden}, 2048, T), ws({kMlp, kMlp}, kHidden, T),
                     ws({kHidden}, kMlp, T), ws({kQProj, 512, 512}, kHidden, T)})
      s->p_gws_bytes = std::max(s->p_gws_bytes, w);
  struct Part {
    void** p;
    size_t bytes;
  } parts[] = {
      {(void**)&s->p_h, N * kHidden * 2},          {(void**)&s->p_xn, N * kHidden * 2},
      {(void**)&s->p_raw, N * kGdnConv * 2},       {(void**)&s->p_z, N * 2048 * 2},
      {(void**)&s->p_ab, N * 32 * 2},              {(void**)&s->p_conv, N * kGdnConv * 2},
      {(void**)&s->p_y, N * 2048 * 2},             {(void**)&s->p_gated, N * 2048 * 2},
      {(void**)&s->p_q, N * kQProj * 2},           {(void**)&s->p_k, N * 512 * 2},
      {(void**)&s->p_v, N * 512 * 2},              {(void**)&s->p_gu, 2 * N * kMlp * 2},
      {(void**)&s->p_act, N * kMlp * 2},           {(void**)&s->p_qn, 8 * N * 256 * 2},
      {(void**)&s->p_zs, N * 2048 * 4},            {(void**)&s->p_rope, N * 64 * 4},
      {(void**)&s->p_kq, 16 * N * 256 * 4},        {(void**)&s->p_gb, 16 * N * 2 * 4},
      {(void**)&s->p_vv, 16 * 8 * N * 16 * 4},     {(void**)&s->p_opart, items * 128 * 256 * 4},
      {(void**)&s->p_oml, items * 128 * 2 * 4},    {(void**)&s->p_gws, s->p_gws_bytes},
      {(void**)&s->p_omax, items * 128 * 4},
  };
  size_t total = 0;
  for (auto& pt : parts) total += (pt.bytes + 255) & ~size_t(255);
  cudaError_t e = cudaMalloc(&s->pbuf, total);
  if (e == cudaSuccess) e = cudaMemset(s->pbuf, 0, total);
  if (e != cudaSuccess) {
    if (s->pbuf) cudaFree(s->pbuf);
    s->pbuf = nullptr;
    return e;
  }
  size_t off = 0;
  for (auto& pt : parts) {
    *pt.p = s->pbuf + off;
    off += (pt.bytes + 255) & ~size_t(255);
  }
  return cudaSuccess;
}

// One prompt chunk on the tensor cores: tokens p0 .. p0 + T - 1 (seq on the
// device) through all 24 layers without the head, in the order of the
// reference's prefill layer body (model.rs:233-289): per layer the input norm,
// the fused projections as one GEMM over the chunk, the GDN conv, preparation
// and recurrence (or the attention preparation, flash attention and gate),
// the output projection with the residual, then the MLP.
cudaError_t enqueue_prompt_chunk(q35_session* s, uint32_t p0, int T) {
  const ModelW& M = s->M;
  cudaStream_t st = s->stream;
  bool pdl = false;
  cudaError_t e = cudaSuccess;
#define Q35_P(x)                    \
  do {                              \
    e = (x);                        \
    if (e != cudaSuccess) return e; \
    pdl = true;                     \
  } while (0)
  auto gemm = [&](const uint16_t* x, int K, std::initializer_list<QGemmSeg> segs) {
    QGemmArgs g = {};
    int i = 0;
    for (const QGemmSeg& sg : segs) g.seg[i++] = sg;
    g.nseg = i;
    g.x = x;
    g.K = K;
    g.T = T;
    g.err = &s->ctl->err;
    return launch_qgemm(g, s->p_gws, s->p_gws_bytes, false, st, pdl);
  };
  auto rms = [&](const uint16_t* gain, bool embed) {
    TokArgs t = {};
    t.n = T;
    t.h_in = s->p_h;
    t.gain = gain;
    t.xn = s->p_xn;
    if (embed) {
      t.ew = M.embed.w;
      t.es = M.embed.s;
      t.eb = M.embed.b;
      t.h_out = s->p_h;
      t.seq = s->seq;
      t.p0 = p0;
      t.ctl = s->ctl;
      t.rope = s->p_rope;
    }
    return launch_tok_rms(t, st, pdl);
  };
  PromptArgs pa = {};
  pa.T = T;
  pa.p0 = p0;
  pa.tmax = s->prompt_chunk;
  pa.ctl = s->ctl;
  pa.raw = s->p_raw;
  pa.conv = s->p_conv;
  pa.ab = s->p_ab;
  pa.z = s->p_z;
  pa.zs = s->p_zs;
  pa.kq = s->p_kq;
  pa.gb = s->p_gb;
  pa.vv = s->p_vv;
  pa.y = s->p_y;
  pa.q_raw = s->p_q;
  pa.k_raw = s->p_k;
  pa.v_raw = s->p_v;
  pa.rope = s->p_rope;
  pa.qn = s->p_qn;
  pa.capacity = s->capacity;
  pa.opart = s->p_opart;
  pa.oml = s->p_oml;
  pa.omax = s->p_omax;
  pa.gated = s->p_gated;
  prompt_attn_plan(pa);
  int gi = 0, ai = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerW& L = M.L[l];
    Q35_P(rms(L.in_norm, l == 0));
    if (!L.attn) {
      Q35_P(gemm(s->p_xn, kHidden, {{L.qkv.w, L.qkv.s, L.qkv.b, s->p_raw, nullptr, kGdnConv, kGdnConv},
                                    {L.z.w, L.z.s, L.z.b, s->p_z, nullptr, 2048, 2048},
                                    {L.a.w, L.a.s, L.a.b, s->p_ab, nullptr, 16, 32},
                                    {L.bproj.w, L.bproj.s, L.bproj.b, s->p_ab + 16, nullptr, 16, 32}}));
      pa.hist = s->hist + size_t(gi) * 3 * kGdnConv;
      pa.convw = L.conv;
      pa.a_log = L.alog;
      pa.dt_bias = L.dt;
      pa.state = s->state + size_t(gi) * kGdnHeads * 128 * 128;
      Q35_P(launch_prompt_conv(pa, st, pdl));
      Q35_P(launch_prompt_gdn_prep(pa, st, pdl));
      Q35_P(launch_prompt_recur(pa, st, pdl));
      TokArgs g = {};
      g.n = T;
      g.y = s->p_y;
      g.zs = s->p_zs;
      g.gw = L.gnorm;
      g.gated = s->p_gated;
      Q35_P(launch_tok_normgate(g, st, pdl));
      Q35_P(gemm(s->p_gated, 2048, {{L.out.w, L.out.s, L.out.b, s->p_h, s->p_h, kHidden, kHidden}}));
      ++gi;
    } else {
      Q35_P(gemm(s->p_xn, kHidden, {{L.q.w, L.q.s, L.q.b, s->p_q, nullptr, kQProj, kQProj},
                                    {L.k.w, L.k.s, L.k.b, s->p_k, nullptr, 512, 512},
                                    {L.v.w, L.v.s, L.v.b, s->p_v, nullptr, 512, 512}}));
      pa.q_gain = L.qnorm;
      pa.k_gain = L.knorm;
      pa.kcache = s->kcache(ai);
      pa.vcache = s->vcache(ai);
      Q35_P(launch_prompt_attn_prep(pa, st, pdl));
      Q35_P(launch_prompt_attn(pa, st, pdl));
      Q35_P(gemm(s->p_gated, 2048, {{L.o.w, L.o.s, L.o.b, s->p_h, s->p_h, kHidden, kHidden}}));
      ++ai;
    }
    Q35_P(rms(L.post_norm, false));
    Q35_P(gemm(s->p_xn, kHidden, {{L.gate.w, L.gate.s, L.gate.b, s->p_gu, nullptr, kMlp, kMlp},
                                  {L.up.w, L.up.s, L.up.b, s->p_gu + size_t(T) * kMlp, nullptr, kMlp, kMlp}}));
    TokArgs sw = {};
    sw.n = T;
    sw.g = s->p_gu;
    sw.u = s->p_gu + size_t(T) * kMlp;
    sw.act = s->p_act;
    Q35_P(launch_tok_swiglu(sw, st, pdl));
    Q35_P(gemm(s->p_act, kMlp, {{L.down.w, L.down.s, L.down.b, s->p_h, s->p_h, kHidden, kHidden}}));
  }
#undef Q35_P
  return e;
}

// Kernel nodes of a captured graph: the launches one replay performs.
uint32_t kernel_nodes(cudaGraph_t g) {
  size_t n = 0;
  if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || n == 0) return 0;
  std::vector<cudaGraphNode_t> nodes(n);
  if (cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return 0;
  uint32_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
  }
  return k;
}

cudaError_t capture(q35_session* s, int steps, bool head, cudaGraphExec_t* out, uint32_t* knodes = nullptr) {
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return e;
  cudaError_t le = cudaSuccess;
  for (int i = 0; i < steps && le == cudaSuccess; ++i) le = enqueue_step(s, head, i == 0);
  e = cudaStreamEndCapture(s->stream, &g);
  if (le != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return le;
  }
  if (e != cudaSuccess) return e;
  if (knodes) *knodes = kernel_nodes(g);
  e = cudaGraphInstantiate(out, g, 0);
  // upload now, so that the first replay (inside a request or a timed region)
  // does not pay for it
  if (e == cudaSuccess) e = cudaGraphUpload(*out, s->stream);
  cudaGraphDestroy(g);
  return e;
}

void free_session(q35_session* s) {
  if (!s) return;
  if (s->device >= 0) cudaSetDevice(s->device);
  for (cudaGraphExec_t g : {s->gdec1, s->gdecN, s->gpre1, s->gpreN, s->gchunk})
    if (g) cudaGraphExecDestroy(g);
  for (cudaEvent_t ev : s->inflight)
    if (ev) cudaEventDestroy(ev);
  for (void* p : s->xpeer)
    if (p) cudaIpcCloseMemHandle(p);
  if (s->xtab) cudaFree(s->xtab);
  if (s->xbuf) cudaFree(s->xbuf);
  if (s->xkv) cudaFree(s->xkv);
  if (s->buf) cudaFree(s->buf);
  if (s->pbuf) cudaFree(s->pbuf);
  if (s->M.arena) cudaFree(s->M.arena);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

// Device-state reset (Model::reset, model.rs:93-96): GDN state and history
// zeroed, position 0, no pending token.
cudaError_t reset_state(q35_session* s) {
  s->position = 0;
  s->has_pending = false;
  cudaError_t e = cudaMemsetAsync(s->state, 0, size_t(18) * kGdnHeads * 128 * 128 * 4, s->stream);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(s->hist, 0, size_t(18) * 3 * kGdnConv * 2, s->stream);
  return e;
}

int device_failure(q35_session* s, cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  cudaStreamSynchronize(s->stream);
  reset_state(s);
  cudaStreamSynchronize(s->stream);
  return set_err(s, Q35_ECUDA, m);
}

// Runs `n` steps from the current device state (graphs of the batch size
// then single steps). Returns 0, Q35_ECANCEL or a CUDA error code.
// Before the i-th launch of a loop: wait until launch i - kInflight has
// finished, so at most kInflight graph launches (chunks) are queued and a
// cancel waits for no more than that; after it: mark its end.
cudaError_t inflight_wait(q35_session* s, size_t i) {
  return i >= size_t(kInflight) ? cudaEventSynchronize(s->inflight[i % kInflight]) : cudaSuccess;
}
cudaError_t inflight_mark(q35_session* s, size_t i) {
  return cudaEventRecord(s->inflight[i % kInflight], s->stream);
}

int run_steps(q35_session* s, size_t n, bool head, cudaError_t* ce) {
  cudaGraphExec_t g1 = head ? s->gdec1 : s->gpre1;
  cudaGraphExec_t gN = head ? s->gdecN : s->gpreN;
  const size_t B = size_t(head ? s->dbatch : s->pbatch);
  size_t launched = 0;
  while (n > 0) {
    cudaError_t e = inflight_wait(s, launched);
    if (e != cudaSuccess) {
      *ce = e;
      return Q35_ECUDA;
    }
    if (s->cancelled.load(std::memory_order_relaxed)) return Q35_ECANCEL;
    if (!head && s->gchunk && n >= size_t(kPrefillTokens)) {
      e = cudaGraphLaunch(s->gchunk, s->stream);
      n -= kPrefillTokens;
    } else if (n >= B && gN) {
      e = cudaGraphLaunch(gN, s->stream);
      n -= B;
      if (head) s->launches += s->kn_decN;
    } else {
      e = cudaGraphLaunch(g1, s->stream);
      n -= 1;
      if (head) s->launches += s->kn_dec1;
    }
    if (e == cudaSuccess) e = inflight_mark(s, launched++);
    if (e != cudaSuccess) {
      *ce = e;
      return Q35_ECUDA;
    }
  }
  return Q35_OK;
}

// The prompt (positions 0 .. n - 1, already in seq) through tensor-core
// chunks of up to prompt_chunk tokens, enqueued directly (each chunk's shapes
// are known here); the host waits every few chunks so a cancel is observed.
int run_prompt_tensor(q35_session* s, size_t n, cudaError_t* ce) {
  cudaError_t e = ensure_prompt_buffers(s);
  uint32_t p0 = 0;
  size_t queued = 0;
  while (e == cudaSuccess && n > 0) {
    e = inflight_wait(s, queued);
    if (e != cudaSuccess) break;
    if (s->cancelled.load(std::memory_order_relaxed)) return Q35_ECANCEL;
    const int T = int(std::min(n, size_t(s->prompt_chunk)));
    e = enqueue_prompt_chunk(s, p0, T);
    p0 += uint32_t(T);
    n -= size_t(T);
    if (e == cudaSuccess) e = inflight_mark(s, queued++);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) {
    *ce = e;
    return Q35_ECUDA;
  }
  return Q35_OK;
}

// A sequence-split session's prompt on the tensor cores: every rank runs the
// whole prompt route over all n rows in the full-capacity layout (so the GDN
// state and conv history come out identical on every rank), then keeps only
// its own positions p = l G + rank, moved to the local layout the split's
// attention reads (local index l at chain l % 64, slot l / 64, heads at the
// local capacity's stride). One layer at a time goes through a full-capacity
// copy, since both layouts share the cache buffer. For local chain c the
// source positions sit on one global chain, (c G + rank) % 64, every G-th
// slot from (c G + rank) / 64: one strided 2-D copy per (layer, K/V, head,
// chain).
cudaError_t split_keep_local_rows(q35_session* s, size_t n) {
  const size_t G = size_t(s->xworld), R = size_t(s->xrank);
  const size_t cap = s->capacity, cps = cap / kAttnChains;
  const size_t lcap = s->kv_capacity(), lcps = lcap / kAttnChains;
  const size_t nloc = n > R ? (n - R + G - 1) / G : 0;
  const size_t layer_elems = size_t(2) * kKvHeads * cap * kHeadDim;  // K then V, as kcache/vcache lie
  const size_t row = size_t(kHeadDim) * 2;
  cudaError_t e = cudaSuccess;
  if (!s->xkv) e = cudaMalloc(&s->xkv, layer_elems * 2);
  for (int ai = 0; ai < 6 && e == cudaSuccess; ++ai) {
    e = cudaMemcpyAsync(s->xkv, s->kcache(ai), layer_elems * 2, cudaMemcpyDeviceToDevice, s->stream);
    for (int which = 0; which < 2 && e == cudaSuccess; ++which)
      for (int h = 0; h < kKvHeads && e == cudaSuccess; ++h) {
        const uint16_t* src = s->xkv + (size_t(which) * kKvHeads + h) * cap * kHeadDim;
        uint16_t* dst = (which ? s->vcache(ai) : s->kcache(ai)) + size_t(h) * lcap * kHeadDim;
        for (size_t c = 0; c < size_t(kAttnChains) && e == cudaSuccess; ++c) {
          const size_t rows = nloc > c ? (nloc - c + kAttnChains - 1) / kAttnChains : 0;
          if (rows == 0) continue;
          const size_t gc = (c * G + R) % kAttnChains, k0 = (c * G + R) / kAttnChains;
          e = cudaMemcpy2DAsync(dst + c * lcps * kHeadDim, row, src + (gc * cps + k0) * kHeadDim, G * row, row,
                                rows, cudaMemcpyDeviceToDevice, s->stream);
        }
      }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  return e;
}

int check_device_ctl(q35_session* s) {
  Ctl c;
  cudaError_t e = cudaMemcpy(&c, s->ctl, sizeof(Ctl), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return device_failure(s, e, "control read");
  if (c.err != 0) {
    std::string m = c.err == kErrToken   ? std::string("token outside vocabulary on device")
                    : c.err == kErrXWait ? std::string("sequence split: a peer's attention record did not arrive")
                                         : "device wait expired (site " + std::to_string(c.err) + ")";
    reset_state(s);
    cudaStreamSynchronize(s->stream);
    return set_err(s, Q35_ETIMEOUT, m);
  }
  return Q35_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Batched sessions: up to kMaxSessions sessions of one device decoded together.
// Each step streams the weights once for all of them (chunk matvecs over the
// sessions' pending tokens, the batched head), while each session keeps its
// own control block, token ring, GDN state, conv history and KV cache; its
// tokens are those it would produce decoding alone.
// ---------------------------------------------------------------------------
struct q35_batch {
  int n = 0;
  int device = 0;
  bool tensor = false;  // tensor-core route (GEMMs on tcgen05) instead of the exact matvecs
  q35_session* s[kMaxTensorSessions] = {};
  cudaStream_t stream = nullptr;
  uint8_t* buf = nullptr;
  Ctl** ctls = nullptr;
  uint32_t** seqs = nullptr;
  uint16_t** hists = nullptr;
  float** states = nullptr;
  uint16_t *h = nullptr, *conv = nullptr, *z = nullptr, *ab = nullptr, *y = nullptr;
  uint16_t *q = nullptr, *k = nullptr, *v = nullptr, *gated = nullptr, *act = nullptr;
  float *rope = nullptr, *po = nullptr, *pml = nullptr, *zs = nullptr;
  // tensor route: normalised inputs, projection outputs, logits, GEMM
  // workspace, per-session attention and head tables
  uint16_t *xn = nullptr, *raw = nullptr, *gu = nullptr, *logits = nullptr;
  uint8_t* gws = nullptr;
  size_t gws_bytes = 0;
  AttnSess* asess = nullptr;
  HeadOut* hout = nullptr;
  cudaGraphExec_t g1 = nullptr, gN = nullptr;
  uint32_t kn_g1 = 0, kn_gN = 0;  // kernel launches per replay (counted at capture)
  uint64_t launches = 0;          // since the last q35_batch_launch_count reset
  int nbatch = 8;
  std::string err;
};

namespace {

cudaError_t enqueue_batch_step(q35_batch* b, bool first) {
  const ModelW& M = b->s[0]->M;
  cudaStream_t st = b->stream;
  const int n = b->n;
  bool pdl = !first;
  cudaError_t e = cudaSuccess;
#define Q35_B(x)                    \
  do {                              \
    e = (x);                        \
    if (e != cudaSuccess) return e; \
    pdl = true;                     \
  } while (0)
  auto rows = [&](QmvArgs& a) {
    a.ntok = n;
    a.sub = chunk_sub_tokens(a);
    a.ctl = b->s[0]->ctl;
  };
  int gi = 0, ai = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerW& L = M.L[l];
    if (!L.attn) {
      QmvArgs a = {};
      a.seg[0] = {L.qkv.w, L.qkv.s, L.qkv.b, nullptr, 6144};
      a.seg[1] = {L.z.w, L.z.s, L.z.b, b->z, 2048};
      a.seg[2] = {L.a.w, L.a.s, L.a.b, b->ab, 16};
      a.seg[3] = {L.bproj.w, L.bproj.s, L.bproj.b, b->ab + 16, 16};
      a.ystride[1] = 2048;
      a.ystride[2] = 32;
      a.ystride[3] = 32;
      a.nseg = 4;
      a.K = 1024;
      a.units = 8224;
      a.units_per_cta = 56;
      a.pro = l == 0 ? kProEmbedRms : kProRms;
      a.epi = kEpiGdnConv;
      a.x = b->h;
      a.gain = L.in_norm;
      a.h_out = b->h;
      a.ew = M.embed.w;
      a.es = M.embed.s;
      a.eb = M.embed.b;
      a.rope_out = b->rope;
      a.convw = L.conv;
      a.conv_out = b->conv;
      a.sess = 1;
      a.ctls = b->ctls;
      a.seqs = b->seqs;
      a.hists = b->hists;
      a.hist_off = size_t(gi) * 3 * kGdnConv;
      rows(a);
      Q35_B(launch_qmv_chunk(a, st, pdl));
      RecurArgs r = {};
      r.conv = b->conv;
      r.a_raw = b->ab;
      r.b_raw = b->ab + 16;
      r.a_log = L.alog;
      r.dt_bias = L.dt;
      r.y = b->y;
      r.advance_pos = l == 0;
      r.states = b->states;
      r.state_off = size_t(gi) * kGdnHeads * 128 * 128;
      r.ctls = b->ctls;
      r.z = b->z;
      r.zs = b->zs;
      Q35_B(launch_recur_sessions(r, n, st, pdl));
      QmvArgs o = {};
      o.seg[0] = {L.out.w, L.out.s, L.out.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProNormGate;
      o.gy = b->y;
      o.gz = b->z;
      o.gzs = b->zs;
      o.gw = L.gnorm;
      o.epi = kEpiResAdd;
      o.res = b->h;
      rows(o);
      Q35_B(launch_qmv_chunk(o, st, pdl));
      ++gi;
    } else {
      QmvArgs a = {};
      a.seg[0] = {L.q.w, L.q.s, L.q.b, b->q, 4096};
      a.seg[1] = {L.k.w, L.k.s, L.k.b, b->k, 512};
      a.seg[2] = {L.v.w, L.v.s, L.v.b, b->v, 512};
      a.ystride[0] = kQProj;
      a.ystride[1] = 512;
      a.ystride[2] = 512;
      a.nseg = 3;
      a.K = 1024;
      a.units = 5120;
      a.units_per_cta = 36;
      a.pro = kProRms;
      a.x = b->h;
      a.gain = L.in_norm;
      a.epi = kEpiStore;
      rows(a);
      Q35_B(launch_qmv_chunk(a, st, pdl));
      for (int t = 0; t < n; ++t) {
        q35_session* ss = b->s[t];
        AttnArgs at = {};
        at.q_raw = b->q + size_t(t) * kQProj;
        at.k_raw = b->k + size_t(t) * 512;
        at.v_raw = b->v + size_t(t) * 512;
        at.q_gain = L.qnorm;
        at.k_gain = L.knorm;
        at.kcache = ss->kcache(ai);
        at.vcache = ss->vcache(ai);
        at.capacity = ss->capacity;
        at.part_o = b->po;
        at.part_ml = b->pml;
        at.gated = b->gated + size_t(t) * 2048;
        at.ctl = ss->ctl;
        at.rope = b->rope + 64 * t;
        Q35_B(launch_attn(at, st, pdl));
      }
      QmvArgs o = {};
      o.seg[0] = {L.o.w, L.o.s, L.o.b, nullptr, 1024};
      o.nseg = 1;
      o.K = 2048;
      o.units = 1024;
      o.units_per_cta = 7;
      o.pro = kProPlain;
      o.x = b->gated;
      o.epi = kEpiResAdd;
      o.res = b->h;
      rows(o);
      Q35_B(launch_qmv_chunk(o, st, pdl));
      ++ai;
    }
    QmvArgs m = {};
    m.seg[0] = {L.gate.w, L.gate.s, L.gate.b, b->act, kMlp};
    m.seg[1] = {L.up.w, L.up.s, L.up.b, nullptr, kMlp};
    m.ystride[0] = kMlp;
    m.nseg = 2;
    m.K = 1024;
    m.units = kMlp;
    m.units_per_cta = 25;
    m.pro = kProRms;
    m.x = b->h;
    m.gain = L.post_norm;
    m.epi = kEpiSwiglu;
    rows(m);
    Q35_B(launch_qmv_chunk(m, st, pdl));
    QmvArgs d = {};
    d.seg[0] = {L.down.w, L.down.s, L.down.b, nullptr, 1024};
    d.nseg = 1;
    d.K = kMlp;
    d.units = 1024;
    d.units_per_cta = 7;
    d.pro = kProPlain;
    d.x = b->act;
    d.epi = kEpiResAdd;
    d.res = b->h;
    rows(d);
    Q35_B(launch_qmv_chunk(d, st, pdl));
  }
  HeadBatchArgs hb = {};
  hb.w = M.embed.w;
  hb.s = M.embed.s;
  hb.b = M.embed.b;
  hb.x = b->h;
  hb.gain = M.norm;
  hb.n = n;
  for (int t = 0; t < n; ++t) {
    q35_session* ss = b->s[t];
    hb.out[t] = {ss->logits, ss->head_part, ss->seq, ss->out_tokens, ss->capacity + 1, ss->capacity,
                 ss->lse, ss->ctl};
  }
  Q35_B(launch_head_batch(hb, st, pdl));
#undef Q35_B
  return e;
}

// One batched step on the tensor cores: the per-token steps of q35_tokens.cu
// around one multi-segment GEMM per fused projection (q35_gemm.cu), the
// sessions' recurrences and attention in one launch each, the head as a GEMM
// over the vocabulary and a per-session greedy selection.
cudaError_t enqueue_batch_step_tensor(q35_batch* b, bool first) {
  const ModelW& M = b->s[0]->M;
  cudaStream_t st = b->stream;
  const int n = b->n;
  bool pdl = !first;
  cudaError_t e = cudaSuccess;
#define Q35_T(x)                    \
  do {                              \
    e = (x);                        \
    if (e != cudaSuccess) return e; \
    pdl = true;                     \
  } while (0)
  auto gemm = [&](const uint16_t* x, int K, std::initializer_list<QGemmSeg> segs) {
    QGemmArgs g = {};
    int i = 0;
    for (const QGemmSeg& sg : segs) g.seg[i++] = sg;
    g.nseg = i;
    g.x = x;
    g.K = K;
    g.T = n;
    g.err = &b->s[0]->ctl->err;
    return launch_qgemm(g, b->gws, b->gws_bytes, false, st, pdl);
  };
  auto rms = [&](const uint16_t* gain, bool embed) {
    TokArgs t = {};
    t.n = n;
    t.h_in = b->h;
    t.gain = gain;
    t.xn = b->xn;
    if (embed) {
      t.ew = M.embed.w;
      t.es = M.embed.s;
      t.eb = M.embed.b;
      t.h_out = b->h;
      t.ctls = b->ctls;
      t.seqs = b->seqs;
      t.rope = b->rope;
    }
    return launch_tok_rms(t, st, pdl);
  };
  auto mlp = [&](const LayerW& L) -> cudaError_t {
    cudaError_t r = rms(L.post_norm, false);
    if (r != cudaSuccess) return r;
    pdl = true;
    r = gemm(b->xn, kHidden, {{L.gate.w, L.gate.s, L.gate.b, b->gu, nullptr, kMlp, kMlp},
                              {L.up.w, L.up.s, L.up.b, b->gu + size_t(n) * kMlp, nullptr, kMlp, kMlp}});
    if (r != cudaSuccess) return r;
    TokArgs t = {};
    t.n = n;
    t.g = b->gu;
    t.u = b->gu + size_t(n) * kMlp;
    t.act = b->act;
    r = launch_tok_swiglu(t, st, true);
    if (r != cudaSuccess) return r;
    return gemm(b->act, kMlp, {{L.down.w, L.down.s, L.down.b, b->h, b->h, kHidden, kHidden}});
  };
  int gi = 0, ai = 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerW& L = M.L[l];
    Q35_T(rms(L.in_norm, l == 0));
    if (!L.attn) {
      Q35_T(gemm(b->xn, kHidden, {{L.qkv.w, L.qkv.s, L.qkv.b, b->raw, nullptr, kGdnConv, kGdnConv},
                                  {L.z.w, L.z.s, L.z.b, b->z, nullptr, 2048, 2048},
                                  {L.a.w, L.a.s, L.a.b, b->ab, nullptr, 16, 32},
                                  {L.bproj.w, L.bproj.s, L.bproj.b, b->ab + 16, nullptr, 16, 32}}));
      TokArgs c = {};
      c.n = n;
      c.raw = b->raw;
      c.raw_stride = kGdnConv;
      c.conv = b->conv;
      c.hists = b->hists;
      c.hist_off = size_t(gi) * 3 * kGdnConv;
      c.convw = L.conv;
      Q35_T(launch_tok_conv(c, st, pdl));
      RecurArgs r = {};
      r.conv = b->conv;
      r.a_raw = b->ab;
      r.b_raw = b->ab + 16;
      r.a_log = L.alog;
      r.dt_bias = L.dt;
      r.y = b->y;
      r.advance_pos = l == 0;
      r.states = b->states;
      r.state_off = size_t(gi) * kGdnHeads * 128 * 128;
      r.ctls = b->ctls;
      r.z = b->z;
      r.zs = b->zs;
      Q35_T(launch_recur_sessions(r, n, st, pdl));
      TokArgs g = {};
      g.n = n;
      g.y = b->y;
      g.zs = b->zs;
      g.gw = L.gnorm;
      g.gated = b->gated;
      Q35_T(launch_tok_normgate(g, st, pdl));
      Q35_T(gemm(b->gated, 2048, {{L.out.w, L.out.s, L.out.b, b->h, b->h, kHidden, kHidden}}));
      ++gi;
    } else {
      Q35_T(gemm(b->xn, kHidden, {{L.q.w, L.q.s, L.q.b, b->q, nullptr, kQProj, kQProj},
                                  {L.k.w, L.k.s, L.k.b, b->k, nullptr, 512, 512},
                                  {L.v.w, L.v.s, L.v.b, b->v, nullptr, 512, 512}}));
      AttnArgs at = {};
      at.q_raw = b->q;
      at.k_raw = b->k;
      at.v_raw = b->v;
      at.q_gain = L.qnorm;
      at.k_gain = L.knorm;
      at.part_o = b->po;
      at.part_ml = b->pml;
      at.gated = b->gated;
      at.rope = b->rope;
      at.sess = b->asess + size_t(ai) * n;
      at.ctl = b->s[0]->ctl;
      Q35_T(launch_attn_sessions(at, n, st, pdl));
      Q35_T(gemm(b->gated, 2048, {{L.o.w, L.o.s, L.o.b, b->h, b->h, kHidden, kHidden}}));
      ++ai;
    }
    Q35_T(mlp(L));
  }
  Q35_T(rms(M.norm, false));
  Q35_T(gemm(b->xn, kHidden, {{M.embed.w, M.embed.s, M.embed.b, b->logits, nullptr, kVocab, kVocab}}));
  Q35_T(launch_greedy_sessions(b->hout, n, st, pdl));
#undef Q35_T
  return e;
}

cudaError_t capture_batch(q35_batch* b, int steps, cudaGraphExec_t* out, uint32_t* knodes) {
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return e;
  cudaError_t le = cudaSuccess;
  for (int i = 0; i < steps && le == cudaSuccess; ++i)
    le = b->tensor ? enqueue_batch_step_tensor(b, i == 0) : enqueue_batch_step(b, i == 0);
  e = cudaStreamEndCapture(b->stream, &g);
  if (le != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return le;
  }
  if (e != cudaSuccess) return e;
  *knodes = kernel_nodes(g);
  e = cudaGraphInstantiate(out, g, 0);
  // upload now, so that the first replay (inside a request or a timed region)
  // does not pay for it
  if (e == cudaSuccess) e = cudaGraphUpload(*out, b->stream);
  cudaGraphDestroy(g);
  return e;
}

void free_batch(q35_batch* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  for (cudaGraphExec_t g : {b->g1, b->gN})
    if (g) cudaGraphExecDestroy(g);
  if (b->buf) cudaFree(b->buf);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

int batch_err(q35_batch* b, int code, const std::string& m) {
  b->err = m;
  return code;
}

// Runs `steps` batched steps; returns Q35_OK or an error (sessions reset on
// device errors, as single sessions are).
int batch_run(q35_batch* b, size_t steps, float* ms) {
  for (int t = 0; t < b->n; ++t) {
    q35_session* ss = b->s[t];
    if (!ss->has_pending) return batch_err(b, Q35_EINVAL, "session " + std::to_string(t) + ": no continuation state");
    if (ss->position + steps > ss->capacity)
      return batch_err(b, Q35_EINVAL, "session " + std::to_string(t) + ": context capacity exceeded");
  }
  cudaSetDevice(b->device);
  cudaError_t e = cudaSuccess;
  for (int t = 0; t < b->n && e == cudaSuccess; ++t) {
    e = cudaStreamSynchronize(b->s[t]->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(&b->s[t]->ctl->out_count, 0, 4, b->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  cudaEvent_t ea = nullptr, eb = nullptr;
  if (ms) {
    cudaEventCreate(&ea);
    cudaEventCreate(&eb);
    if (e == cudaSuccess) e = cudaEventRecord(ea, b->stream);
  }
  size_t left = steps, launched = 0;
  while (left > 0 && e == cudaSuccess) {
    if (left >= size_t(b->nbatch) && b->gN) {
      e = cudaGraphLaunch(b->gN, b->stream);
      left -= size_t(b->nbatch);
      b->launches += b->kn_gN;
    } else {
      e = cudaGraphLaunch(b->g1, b->stream);
      left -= 1;
      b->launches += b->kn_g1;
    }
    if (!ms && e == cudaSuccess && ++launched % 16 == 0) e = cudaStreamSynchronize(b->stream);
  }
  if (ms) {
    if (e == cudaSuccess) e = cudaEventRecord(eb, b->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(eb);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, ea, eb);
    cudaEventDestroy(ea);
    cudaEventDestroy(eb);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
  if (e != cudaSuccess) {
    const std::string m = std::string("batched decode: ") + cudaGetErrorString(e);
    for (int t = 0; t < b->n; ++t) device_failure(b->s[t], e, "batched decode");
    return batch_err(b, Q35_ECUDA, m);
  }
  if (b->tensor) {  // each member's last logits into its own buffer (q35_last_logits)
    for (int t = 0; t < b->n && e == cudaSuccess; ++t)
      e = cudaMemcpyAsync(b->s[t]->logits, b->logits + size_t(t) * kVocab, size_t(kVocab) * 2,
                          cudaMemcpyDeviceToDevice, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) {
      for (int t = 0; t < b->n; ++t) device_failure(b->s[t], e, "batched decode");
      return batch_err(b, Q35_ECUDA, std::string("batched decode: ") + cudaGetErrorString(e));
    }
  }
  int rc = Q35_OK;
  for (int t = 0; t < b->n; ++t) {
    const int r = check_device_ctl(b->s[t]);
    if (r != Q35_OK && rc == Q35_OK) {
      rc = r;
      b->err = "session " + std::to_string(t) + ": " + b->s[t]->err;
    }
  }
  return rc;
}

}  // namespace

extern "C" {

const char* q35_version(void) { return "q35-b200 0.1 (sm_100a)"; }

int q35_batch_create(q35_session** sessions, int n, q35_batch** out, char* errbuf, size_t err_len) {
  return q35_batch_create_ex(sessions, n, 0u, out, errbuf, err_len);
}

int q35_batch_create_ex(q35_session** sessions, int n, uint32_t flags, q35_batch** out, char* errbuf,
                        size_t err_len) {
  if (!out) return Q35_EINVAL;
  *out = nullptr;
  auto fail = [&](int code, const std::string& m) {
    copy_err(errbuf, err_len, m);
    return code;
  };
  const bool tensor = (flags & Q35_BATCH_TENSOR_CORES) != 0;
  if (flags & ~uint32_t(Q35_BATCH_TENSOR_CORES)) return fail(Q35_EINVAL, "unknown batch flags");
  if (!sessions || n < 1 || n > (tensor ? kMaxTensorSessions : kMaxSessions))
    return fail(Q35_EINVAL, tensor ? "tensor-core batch needs 1..64 sessions" : "batch needs 1..8 sessions");
  for (int t = 0; t < n; ++t) {
    if (!sessions[t]) return fail(Q35_EINVAL, "null session");
    if (sessions[t]->device != sessions[0]->device) return fail(Q35_EINVAL, "sessions on different devices");
    if (sessions[t]->model_id != sessions[0]->model_id) return fail(Q35_EINVAL, "sessions of different models");
    if (sessions[t]->xworld > 1) return fail(Q35_EINVAL, "sequence-split sessions cannot be batched");
    for (int u = 0; u < t; ++u)
      if (sessions[u] == sessions[t]) return fail(Q35_EINVAL, "session listed twice");
  }
  q35_batch* b = new q35_batch();
  b->n = n;
  b->tensor = tensor;
  b->device = sessions[0]->device;
  for (int t = 0; t < n; ++t) b->s[t] = sessions[t];
  cudaSetDevice(b->device);
  cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  struct Part {
    void** p;
    size_t bytes;
  };
  const size_t N = size_t(n);
  std::vector<Part> parts = {
      {(void**)&b->ctls, 8 * N}, {(void**)&b->seqs, 8 * N}, {(void**)&b->hists, 8 * N},
      {(void**)&b->states, 8 * N}, {(void**)&b->h, N * kHidden * 2}, {(void**)&b->conv, N * kGdnConv * 2},
      {(void**)&b->z, N * 2048 * 2}, {(void**)&b->ab, N * 32 * 2}, {(void**)&b->y, N * 2048 * 2},
      {(void**)&b->q, N * kQProj * 2}, {(void**)&b->k, N * 512 * 2}, {(void**)&b->v, N * 512 * 2},
      {(void**)&b->gated, N * 2048 * 2}, {(void**)&b->act, N * kMlp * 2}, {(void**)&b->rope, N * 64 * 4},
      {(void**)&b->zs, N * 2048 * 4},
      {(void**)&b->po, (tensor ? N : 1) * kKvHeads * kAttnChains * 4 * kHeadDim * 4},
      {(void**)&b->pml, (tensor ? N : 1) * kKvHeads * kAttnChains * 4 * 2 * 4},
  };
  if (tensor) {
    // the largest GEMM workspace of the step (split partials + counters)
    const ModelW& M = sessions[0]->M;
    (void)M;
    auto ws = [&](std::initializer_list<int> rows, int K) {
      QGemmArgs g = {};
      for (int r : rows) g.seg[g.nseg++].rows = r;
      g.K = K;
      g.T = n;
      return qgemm_workspace_bytes(g);
    };
    for (size_t w : {ws({kGdnConv, 2048, 16, 16}, kHidden), ws({kHidden}, 2048), ws({kMlp, kMlp}, kHidden),
                     ws({kHidden}, kMlp), ws({kQProj, 512, 512}, kHidden), ws({kVocab}, kHidden)})
      b->gws_bytes = std::max(b->gws_bytes, w);
    parts.push_back({(void**)&b->xn, N * kHidden * 2});
    parts.push_back({(void**)&b->raw, N * kGdnConv * 2});
    parts.push_back({(void**)&b->gu, 2 * N * kMlp * 2});
    parts.push_back({(void**)&b->logits, N * kVocab * 2});
    parts.push_back({(void**)&b->gws, b->gws_bytes});
    parts.push_back({(void**)&b->asess, 6 * N * sizeof(AttnSess)});
    parts.push_back({(void**)&b->hout, N * sizeof(HeadOut)});
  }
  size_t total = 0;
  for (auto& pt : parts) total += (pt.bytes + 255) & ~size_t(255);
  if (e == cudaSuccess) e = cudaMalloc(&b->buf, total);
  if (e == cudaSuccess) e = cudaMemset(b->buf, 0, total);
  if (e != cudaSuccess) {
    free_batch(b);
    return fail(Q35_ENOMEM, std::string("batch buffers: ") + cudaGetErrorString(e));
  }
  size_t off = 0;
  for (auto& pt : parts) {
    *pt.p = b->buf + off;
    off += (pt.bytes + 255) & ~size_t(255);
  }
  Ctl* hc[kMaxTensorSessions];
  uint32_t* hs[kMaxTensorSessions];
  uint16_t* hh[kMaxTensorSessions];
  float* hst[kMaxTensorSessions];
  for (int t = 0; t < n; ++t) {
    hc[t] = sessions[t]->ctl;
    hs[t] = sessions[t]->seq;
    hh[t] = sessions[t]->hist;
    hst[t] = sessions[t]->state;
  }
  e = cudaMemcpy(b->ctls, hc, 8 * N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->seqs, hs, 8 * N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->hists, hh, 8 * N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->states, hst, 8 * N, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && tensor) {
    std::vector<AttnSess> as(6 * N);
    std::vector<HeadOut> ho(N);
    for (int t = 0; t < n; ++t) {
      q35_session* ss = sessions[t];
      for (int ai = 0; ai < 6; ++ai) as[size_t(ai) * N + t] = {ss->kcache(ai), ss->vcache(ai), ss->ctl, ss->kv_capacity()};
      ho[t] = {b->logits + size_t(t) * kVocab, ss->head_part, ss->seq, ss->out_tokens, ss->capacity + 1, ss->capacity,
               ss->lse, ss->ctl};
    }
    e = cudaMemcpy(b->asess, as.data(), as.size() * sizeof(AttnSess), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(b->hout, ho.data(), ho.size() * sizeof(HeadOut), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = capture_batch(b, 1, &b->g1, &b->kn_g1);
  if (e == cudaSuccess) e = capture_batch(b, b->nbatch, &b->gN, &b->kn_gN);
  if (e != cudaSuccess) {
    free_batch(b);
    return fail(Q35_ECUDA, std::string("batch graph capture: ") + cudaGetErrorString(e));
  }
  *out = b;
  return Q35_OK;
}

int q35_batch_decode(q35_batch* b, size_t steps, uint32_t* out_tokens) {
  if (!b || !out_tokens || steps == 0) return Q35_EINVAL;
  int rc = batch_run(b, steps, nullptr);
  if (rc != Q35_OK) return rc;
  for (int t = 0; t < b->n; ++t) {
    q35_session* ss = b->s[t];
    cudaError_t e = cudaMemcpy(out_tokens + size_t(t) * steps, ss->out_tokens, steps * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return batch_err(b, device_failure(ss, e, "token read"), "token read");
    ss->position += uint32_t(steps);
    ss->pending = out_tokens[size_t(t) * steps + steps - 1];
  }
  return Q35_OK;
}

int q35_batch_decode_timed(q35_batch* b, size_t steps, float* ms) {
  if (!b || !ms || steps == 0) return Q35_EINVAL;
  int rc = batch_run(b, steps, ms);
  if (rc != Q35_OK) return rc;
  for (int t = 0; t < b->n; ++t) {
    q35_session* ss = b->s[t];
    uint32_t last = 0;
    cudaError_t e = cudaMemcpy(&last, ss->out_tokens + (steps - 1), 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return batch_err(b, device_failure(ss, e, "token read"), "token read");
    ss->position += uint32_t(steps);
    ss->pending = last;
  }
  return Q35_OK;
}

const char* q35_batch_last_error(const q35_batch* b) { return b ? b->err.c_str() : "no batch"; }

int q35_batch_launch_count(q35_batch* b, int reset, uint64_t* launches) {
  if (!b) return Q35_EINVAL;
  if (launches) *launches = b->launches;
  if (reset) b->launches = 0;
  return Q35_OK;
}

void q35_batch_destroy(q35_batch* b) { free_batch(b); }

int q35_force_pending(q35_session* s, uint32_t token) {
  if (!s) return Q35_EINVAL;
  if (!s->has_pending) return set_err(s, Q35_EINVAL, "no continuation state");
  if (token >= uint32_t(kVocab)) return set_err(s, Q35_EINVAL, "token outside vocabulary");
  cudaSetDevice(s->device);
  // the next continuation's first step embeds seq[position]
  cudaError_t e = cudaMemcpyAsync(s->seq + s->position, &token, 4, cudaMemcpyHostToDevice, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return device_failure(s, e, "force pending");
  s->pending = token;
  return Q35_OK;
}

int q35_split_prepare(q35_session* s, int rank, int world, void* handle) {
  if (!s || !handle) return Q35_EINVAL;
  if (world < 2 || world > kMaxSplit || rank < 0 || rank >= world)
    return set_err(s, Q35_EINVAL, "split: world must be 2..8 and rank in [0, world)");
  if (s->xworld > 1 || s->xbuf) return set_err(s, Q35_EINVAL, "split: already prepared");
  cudaSetDevice(s->device);
  const size_t bytes = x_recv_bytes(world) + x_flag_bytes(world);
  cudaError_t e = cudaMalloc(&s->xbuf, bytes);
  if (e == cudaSuccess) e = cudaMemset(s->xbuf, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, s->xbuf);
  if (e != cudaSuccess) {
    if (s->xbuf) cudaFree(s->xbuf);
    s->xbuf = nullptr;
    return set_err(s, Q35_ECUDA, std::string("split: exchange buffer: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == Q35_SPLIT_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  s->xrank = rank;
  s->xpend_world = world;
  return Q35_OK;
}

int q35_split_connect(q35_session* s, const void* handles) {
  if (!s || !handles) return Q35_EINVAL;
  if (!s->xbuf || s->xpend_world < 2 || s->xworld > 1) return set_err(s, Q35_EINVAL, "split: prepare first");
  const int G = s->xpend_world;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  std::vector<void*> base(G, nullptr);
  for (int p = 0; p < G && e == cudaSuccess; ++p) {
    if (p == s->xrank) {
      base[p] = s->xbuf;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(handles) + size_t(p) * Q35_SPLIT_HANDLE_BYTES, sizeof(h));
    e = cudaIpcOpenMemHandle(&base[p], h, cudaIpcMemLazyEnablePeerAccess);
    if (e == cudaSuccess) s->xpeer.push_back(base[p]);
  }
  std::vector<void*> tab(2 * G);
  for (int p = 0; p < G; ++p) {
    tab[p] = base[p];
    tab[G + p] = static_cast<uint8_t*>(base[p]) + x_recv_bytes(G);
  }
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&s->xtab), 2 * G * sizeof(void*));
  if (e == cudaSuccess) e = cudaMemcpy(s->xtab, tab.data(), 2 * G * sizeof(void*), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("split: peer mapping: ") + cudaGetErrorString(e));
  // the graphs bake the attention arguments: capture them again with the split
  s->xworld = G;
  for (cudaGraphExec_t* g : {&s->gdec1, &s->gdecN, &s->gpre1, &s->gpreN, &s->gchunk})
    if (*g) {
      cudaGraphExecDestroy(*g);
      *g = nullptr;
    }
  e = capture(s, 1, true, &s->gdec1, &s->kn_dec1);
  if (e == cudaSuccess && s->dbatch > 1) e = capture(s, s->dbatch, true, &s->gdecN, &s->kn_decN);
  if (e == cudaSuccess) e = capture(s, 1, false, &s->gpre1);
  if (e == cudaSuccess && s->pbatch > 1) e = capture(s, s->pbatch, false, &s->gpreN);
  if (e == cudaSuccess && s->chunked) e = capture_chunk(s, &s->gchunk);
  if (e == cudaSuccess) e = reset_state(s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("split: graph capture: ") + cudaGetErrorString(e));
  return Q35_OK;
}

int q35_split_world(const q35_session* s) { return s ? s->xworld : 0; }

int q35_split_set_wait(q35_session* s, uint32_t ms) {
  if (!s) return Q35_EINVAL;
  if (ms < 1 || ms > 600000) return set_err(s, Q35_EINVAL, "split: wait bound must be 1..600000 ms");
  if (s->xworld > 1) return set_err(s, Q35_EINVAL, "split: set the wait bound before connecting");
  s->xwait_ms = ms;
  return Q35_OK;
}

int q35_diag_bounded_wait(uint32_t polls, uint32_t* err_dev, void* stream) {
  if (!err_dev || polls == 0) return Q35_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(err_dev, 0, sizeof(uint32_t), st);
  if (e == cudaSuccess) e = launch_wait_probe(polls, err_dev, st);
  uint32_t site = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&site, err_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return Q35_ECUDA;
  return site == 0 ? Q35_OK : Q35_ETIMEOUT;
}

int q35_diag_inject_device_error(q35_session* s, uint32_t site) {
  if (!s || site == 0) return Q35_EINVAL;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e == cudaSuccess) e = cudaMemcpy(&s->ctl->err, &site, sizeof(uint32_t), cudaMemcpyHostToDevice);
  return e == cudaSuccess ? Q35_OK : Q35_ECUDA;
}

int q35_open(const char* model_dir, int device, const q35_opts* opts, q35_session** out,
             char* errbuf, size_t err_len) {
  if (!out) return Q35_EINVAL;
  *out = nullptr;
  if (!model_dir) {
    copy_err(errbuf, err_len, "--model MODEL_DIR required");
    return Q35_EINVAL;
  }
  q35_session* s = new q35_session();
  s->device = device;
  {
    char* rp = realpath(model_dir, nullptr);
    s->model_id = rp ? rp : model_dir;
    free(rp);
  }
  {
    std::string m;
    if (!validate_opts(opts, m)) {
      copy_err(errbuf, err_len, m);
      delete s;
      return Q35_EINVAL;
    }
  }
  if (opts) {
    if (opts->capacity) s->capacity = opts->capacity;
    if (opts->decode_batch) s->dbatch = int(opts->decode_batch);
    if (opts->prefill_batch) s->pbatch = int(opts->prefill_batch);
    if (opts->flags & Q35_FLAG_TOKEN_BY_TOKEN_PROMPT) s->chunked = false;
    if (opts->flags & Q35_FLAG_TENSOR_PROMPT) s->tensor_prompt = true;
    if (opts->prompt_chunk) s->prompt_chunk = int(opts->prompt_chunk);
  }
  auto fail = [&](int code, const std::string& m) {
    copy_err(errbuf, err_len, m);
    free_session(s);
    return code;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  e = ensure_kernels_init();
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("kernel setup: ") + cudaGetErrorString(e));
  e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("stream: ") + cudaGetErrorString(e));
  for (cudaEvent_t& ev : s->inflight)
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("event: ") + cudaGetErrorString(e));
  {
    Loader ld;
    if (!ld.open(model_dir) || !ld.upload(s->M) || !bind_model(ld, s->M))
      return fail(Q35_EIO, ld.err);
  }
  // scratch, state, caches
  const size_t cap = s->capacity;
  struct Part {
    void** p;
    size_t bytes;
  };
  std::vector<Part> parts = {
      {(void**)&s->ctl, sizeof(Ctl)},
      {(void**)&s->h, kHidden * 2},
      {(void**)&s->conv_out, kGdnConv * 2},
      {(void**)&s->z, 2048 * 2},
      {(void**)&s->ab, 32 * 2},
      {(void**)&s->y, 2048 * 2},
      {(void**)&s->q, kQProj * 2},
      {(void**)&s->k, 512 * 2},
      {(void**)&s->v, 512 * 2},
      {(void**)&s->gated, 2048 * 2},
      {(void**)&s->act, kMlp * 2},
      {(void**)&s->logits, size_t(kVocab) * 2},
      {(void**)&s->lse, 16},
      {(void**)&s->attn_po, size_t(kKvHeads) * kAttnChains * 4 * kHeadDim * 4},
      {(void**)&s->attn_pml, size_t(kKvHeads) * kAttnChains * 4 * 2 * 4},
      {(void**)&s->head_part, size_t(kHeadCtas) * 2 * 4},
      {(void**)&s->zs, 2048 * 4},
      {(void**)&s->seq, (cap + 1) * 4},
      {(void**)&s->out_tokens, cap * 4},
      {(void**)&s->state, size_t(18) * kGdnHeads * 128 * 128 * 4},
      {(void**)&s->hist, size_t(18) * 3 * kGdnConv * 2},
      {(void**)&s->kv, size_t(6) * 2 * kKvHeads * cap * kHeadDim * 2},
      {(void**)&s->c_h, size_t(kPrefillTokens) * kHidden * 2},
      {(void**)&s->c_conv, size_t(kPrefillTokens) * kGdnConv * 2},
      {(void**)&s->c_z, size_t(kPrefillTokens) * 2048 * 2},
      {(void**)&s->c_ab, size_t(kPrefillTokens) * 32 * 2},
      {(void**)&s->c_y, size_t(kPrefillTokens) * 2048 * 2},
      {(void**)&s->c_q, size_t(kPrefillTokens) * kQProj * 2},
      {(void**)&s->c_k, size_t(kPrefillTokens) * 512 * 2},
      {(void**)&s->c_v, size_t(kPrefillTokens) * 512 * 2},
      {(void**)&s->c_gated, size_t(kPrefillTokens) * 2048 * 2},
      {(void**)&s->c_act, size_t(kPrefillTokens) * kMlp * 2},
      {(void**)&s->c_rope, size_t(kPrefillTokens) * 64 * 4},
      {(void**)&s->c_zs, size_t(kPrefillTokens) * 2048 * 4},
  };
  size_t total = 0;
  for (auto& p : parts) total += (p.bytes + 255) & ~size_t(255);
  e = cudaMalloc(&s->buf, total);
  if (e != cudaSuccess) return fail(Q35_ENOMEM, "cudaMalloc of " + std::to_string(total) + " bytes failed");
  e = cudaMemset(s->buf, 0, total);
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("memset: ") + cudaGetErrorString(e));
  size_t off = 0;
  for (auto& p : parts) {
    *p.p = s->buf + off;
    off += (p.bytes + 255) & ~size_t(255);
  }
  if (s->tensor_prompt) {  // the prompt route's chunk buffers, so a shortage shows here
    e = ensure_prompt_buffers(s);
    if (e != cudaSuccess) return fail(Q35_ENOMEM, std::string("prompt buffers: ") + cudaGetErrorString(e));
  }
  Ctl c = {};
  c.capacity = s->capacity;
  c.attn_t0 = ~0ull;
  c.qmv_t0 = ~0ull;
  e = cudaMemcpy(s->ctl, &c, sizeof(Ctl), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = capture(s, 1, true, &s->gdec1, &s->kn_dec1);
  if (e == cudaSuccess && s->dbatch > 1) e = capture(s, s->dbatch, true, &s->gdecN, &s->kn_decN);
  if (e == cudaSuccess) e = capture(s, 1, false, &s->gpre1);
  if (e == cudaSuccess && s->pbatch > 1) e = capture(s, s->pbatch, false, &s->gpreN);
  if (e == cudaSuccess && s->chunked) e = capture_chunk(s, &s->gchunk);
  if (e != cudaSuccess) return fail(Q35_ECUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  *out = s;
  return Q35_OK;
}

void q35_close(q35_session* s) { free_session(s); }

void q35_cancel(q35_session* s) {
  if (s) s->cancelled.store(true, std::memory_order_relaxed);
}

const char* q35_last_error(const q35_session* s) { return s ? s->err.c_str() : "no session"; }

uint32_t q35_position(const q35_session* s) { return s ? s->position : 0; }

uint32_t q35_capacity(const q35_session* s) { return s ? s->capacity : 0; }

int q35_pending(const q35_session* s, uint32_t* token) {
  if (!s || !token) return Q35_EINVAL;
  if (!s->has_pending) return Q35_EINVAL;
  *token = s->pending;
  return Q35_OK;
}

int q35_check_opts(const q35_opts* opts, char* errbuf, size_t err_len) {
  std::string m;
  if (validate_opts(opts, m)) return Q35_OK;
  copy_err(errbuf, err_len, m);
  return Q35_EINVAL;
}

int q35_launch_count(q35_session* s, int reset, uint64_t* launches) {
  if (!s) return Q35_EINVAL;
  if (launches) *launches = s->launches;
  if (reset) s->launches = 0;
  return Q35_OK;
}

// Model::generate + Model::decode (model.rs:97-180)
int q35_generate(q35_session* s, const uint32_t* prompt, size_t n_prompt, size_t max_tokens,
                 int reset, uint32_t* out_tokens) {
  if (!s) return Q35_EINVAL;
  const size_t cap = s->capacity;
  if (max_tokens == 0 || max_tokens > cap) return set_err(s, Q35_EINVAL, "invalid output length");
  if (!out_tokens) return set_err(s, Q35_EINVAL, "output buffer required");
  if (s->cancelled.load()) return set_err(s, Q35_ECANCEL, "input disconnected");
  cudaSetDevice(s->device);
  if (reset) {
    if (n_prompt == 0 || !prompt) return set_err(s, Q35_EINVAL, "reset needs nonempty prompt");
    if (n_prompt + max_tokens - 1 > cap) return set_err(s, Q35_EINVAL, "context capacity exceeded");
    for (size_t i = 0; i < n_prompt; ++i)
      if (prompt[i] >= uint32_t(kVocab)) return set_err(s, Q35_EINVAL, "token outside vocabulary");
  } else {
    if (n_prompt != 0) return set_err(s, Q35_EINVAL, "continuation prompt must be empty");
    if (s->position + max_tokens > cap) return set_err(s, Q35_EINVAL, "context capacity exceeded");
    if (!s->has_pending) return set_err(s, Q35_EINVAL, "no continuation state");
  }
  cudaError_t e = cudaSuccess;
  if (reset) {
    e = reset_state(s);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(s->seq, prompt, n_prompt * 4, cudaMemcpyHostToDevice, s->stream);
    Ctl c = {};
    c.capacity = s->capacity;
    c.attn_t0 = ~0ull;
    c.qmv_t0 = ~0ull;
    c.epoch = ++s->epoch;  // ranks of a sequence split reset in step, so epochs agree
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->ctl, &c, sizeof(Ctl), cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return device_failure(s, e, "reset");
    // the tensor-core prompt route computes every K/V row on this device; a
    // sequence-split rank then keeps its own share
    int rc = s->tensor_prompt ? run_prompt_tensor(s, n_prompt - 1, &e) : run_steps(s, n_prompt - 1, false, &e);
    if (rc == Q35_OK && s->tensor_prompt && s->xworld > 1) {
      e = split_keep_local_rows(s, n_prompt - 1);
      if (e != cudaSuccess) rc = Q35_ECUDA;
    }
    if (rc == Q35_ECANCEL) {
      cudaStreamSynchronize(s->stream);
      reset_state(s);
      cudaStreamSynchronize(s->stream);
      return set_err(s, Q35_ECANCEL, "input disconnected");
    }
    if (rc != Q35_OK) return device_failure(s, e, "prefill");
  } else {
    e = cudaMemsetAsync(&s->ctl->out_count, 0, 4, s->stream);
    if (e != cudaSuccess) return device_failure(s, e, "continue");
  }
  int rc = run_steps(s, max_tokens, true, &e);
  if (rc == Q35_ECANCEL) {
    cudaStreamSynchronize(s->stream);
    reset_state(s);
    cudaStreamSynchronize(s->stream);
    return set_err(s, Q35_ECANCEL, "input disconnected");
  }
  if (rc != Q35_OK) return device_failure(s, e, "decode");
  e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return device_failure(s, e, "decode");
  rc = check_device_ctl(s);
  if (rc != Q35_OK) return rc;
  e = cudaMemcpy(out_tokens, s->out_tokens, max_tokens * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return device_failure(s, e, "token read");
  if (s->cancelled.load()) {
    reset_state(s);
    cudaStreamSynchronize(s->stream);
    return set_err(s, Q35_ECANCEL, "input disconnected");
  }
  s->position = uint32_t(reset ? n_prompt - 1 + max_tokens : s->position + max_tokens);
  s->pending = out_tokens[max_tokens - 1];
  s->has_pending = true;
  return Q35_OK;
}

int q35_decode_timed(q35_session* s, size_t steps, float* ms) {
  if (!s || !ms || steps == 0) return Q35_EINVAL;
  if (!s->has_pending) return set_err(s, Q35_EINVAL, "no continuation state");
  if (s->position + steps > s->capacity) return set_err(s, Q35_EINVAL, "context capacity exceeded");
  cudaSetDevice(s->device);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaError_t e = cudaMemsetAsync(&s->ctl->out_count, 0, 4, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e == cudaSuccess) e = cudaEventRecord(a, s->stream);
  int rc = Q35_OK;
  if (e == cudaSuccess) {
    // no intermediate synchronisation inside the timed region
    cudaGraphExec_t gN = s->gdecN, g1 = s->gdec1;
    size_t n = steps;
    while (n > 0 && e == cudaSuccess) {
      if (n >= size_t(s->dbatch) && gN) {
        e = cudaGraphLaunch(gN, s->stream);
        n -= size_t(s->dbatch);
        s->launches += s->kn_decN;
      } else {
        e = cudaGraphLaunch(g1, s->stream);
        n -= 1;
        s->launches += s->kn_dec1;
      }
    }
  }
  if (e == cudaSuccess) e = cudaEventRecord(b, s->stream);
  if (e == cudaSuccess) e = cudaEventSynchronize(b);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return device_failure(s, e, "timed decode");
  rc = check_device_ctl(s);
  if (rc != Q35_OK) return rc;
  uint32_t last = 0;
  e = cudaMemcpy(&last, s->out_tokens + (steps - 1), 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return device_failure(s, e, "token read");
  s->position += uint32_t(steps);
  s->pending = last;
  return Q35_OK;
}

int q35_attn_timing(q35_session* s, int reset, double* total_us, uint32_t* launches) {
  if (!s) return Q35_EINVAL;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  Ctl c;
  if (e == cudaSuccess) e = cudaMemcpy(&c, s->ctl, sizeof(Ctl), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("timing: ") + cudaGetErrorString(e));
  if (total_us) *total_us = double(c.attn_ns) * 1e-3;
  if (launches) *launches = c.attn_launches;
  if (reset >= 0) {
    c.timing_on = reset > 0 ? 1u : 0u;
    c.attn_done = 0;
    c.attn_launches = 0;
    c.attn_t0 = ~0ull;
    c.attn_ns = 0;
    c.qmv_done = 0;
    c.qmv_launches = 0;
    c.qmv_t0 = ~0ull;
    c.qmv_ns = 0;
    c.qmv_bytes = 0;
    c.attn_tend = 0;
    c.qmv_tend = 0;
    e = cudaMemcpy(s->ctl, &c, sizeof(Ctl), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("timing: ") + cudaGetErrorString(e));
  }
  return Q35_OK;
}

int q35_qmv_timing(q35_session* s, double* total_us, uint32_t* launches, double* weight_bytes) {
  if (!s) return Q35_EINVAL;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  Ctl c;
  if (e == cudaSuccess) e = cudaMemcpy(&c, s->ctl, sizeof(Ctl), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("timing: ") + cudaGetErrorString(e));
  if (total_us) *total_us = double(c.qmv_ns) * 1e-3;
  if (launches) *launches = c.qmv_launches;
  if (weight_bytes) *weight_bytes = double(c.qmv_bytes);
  return Q35_OK;
}

int q35_dump_state(q35_session* s, uint16_t* kv, float* state, uint16_t* hist) {
  if (!s) return Q35_EINVAL;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  const size_t pos = s->position;
  // the caches are chain-major (local index i at chain i % 64, slot i / 64);
  // under a sequence split local index i holds position i * G + rank and the
  // other positions are left zero
  const size_t G = size_t(s->xworld), R = size_t(s->xrank);
  const size_t cap = s->kv_capacity();
  const size_t cps = cap / kAttnChains;
  const size_t nloc = pos > R ? (pos - R + G - 1) / G : 0;
  const size_t slots = (nloc + kAttnChains - 1) / kAttnChains;
  std::vector<uint16_t> tmp(slots * kHeadDim);
  if (kv && G > 1) std::memset(kv, 0, size_t(6) * 2 * kKvHeads * pos * kHeadDim * 2);
  for (int ai = 0; ai < 6 && e == cudaSuccess && kv; ++ai)
    for (int which = 0; which < 2 && e == cudaSuccess; ++which)
      for (int h = 0; h < kKvHeads && e == cudaSuccess; ++h) {
        const uint16_t* src = (which ? s->vcache(ai) : s->kcache(ai)) + size_t(h) * cap * kHeadDim;
        uint16_t* dst = kv + ((size_t(ai) * 2 + which) * kKvHeads + h) * pos * kHeadDim;
        for (size_t c = 0; c < size_t(kAttnChains) && e == cudaSuccess; ++c) {
          const size_t n = nloc > c ? (nloc - c + kAttnChains - 1) / kAttnChains : 0;
          if (n == 0) continue;
          e = cudaMemcpy(tmp.data(), src + c * cps * kHeadDim, n * kHeadDim * 2, cudaMemcpyDeviceToHost);
          for (size_t sl = 0; sl < n; ++sl)
            std::memcpy(dst + ((sl * kAttnChains + c) * G + R) * kHeadDim, tmp.data() + sl * kHeadDim,
                        kHeadDim * 2);
        }
      }
  if (e == cudaSuccess && state)
    e = cudaMemcpy(state, s->state, size_t(18) * kGdnHeads * 128 * 128 * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && hist)
    e = cudaMemcpy(hist, s->hist, size_t(18) * 3 * kGdnConv * 2, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("dump: ") + cudaGetErrorString(e));
  return Q35_OK;
}

int q35_session_copy(q35_session* dst, q35_session* src) {
  if (!dst || !src || dst == src) return Q35_EINVAL;
  if (dst->device != src->device) return set_err(dst, Q35_EINVAL, "copy: sessions on different devices");
  if (dst->model_id != src->model_id) return set_err(dst, Q35_EINVAL, "copy: sessions of different models");
  if (dst->capacity != src->capacity) return set_err(dst, Q35_EINVAL, "copy: capacities differ");
  if (dst->xworld > 1 || src->xworld > 1) return set_err(dst, Q35_EINVAL, "copy: sequence-split sessions");
  cudaSetDevice(dst->device);
  cudaError_t e = cudaStreamSynchronize(src->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(dst->stream);
  const size_t cap = dst->capacity;
  struct Part {
    void* d;
    const void* s;
    size_t bytes;
  };
  const Part parts[] = {
      {dst->ctl, src->ctl, sizeof(Ctl)},
      {dst->seq, src->seq, (cap + 1) * 4},
      {dst->state, src->state, size_t(18) * kGdnHeads * 128 * 128 * 4},
      {dst->hist, src->hist, size_t(18) * 3 * kGdnConv * 2},
      {dst->kv, src->kv, size_t(6) * 2 * kKvHeads * cap * kHeadDim * 2},
      {dst->logits, src->logits, size_t(kVocab) * 2},
      {dst->lse, src->lse, 2},
  };
  for (const Part& pt : parts)
    if (e == cudaSuccess) e = cudaMemcpyAsync(pt.d, pt.s, pt.bytes, cudaMemcpyDeviceToDevice, dst->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(dst->stream);
  if (e != cudaSuccess) return device_failure(dst, e, "copy");
  dst->position = src->position;
  dst->pending = src->pending;
  dst->has_pending = src->has_pending;
  return Q35_OK;
}

int q35_last_logits(q35_session* s, uint16_t* logits, uint16_t* lse) {
  if (!s) return Q35_EINVAL;
  cudaSetDevice(s->device);
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e == cudaSuccess && logits)
    e = cudaMemcpy(logits, s->logits, size_t(kVocab) * 2, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && lse) e = cudaMemcpy(lse, s->lse, 2, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_err(s, Q35_ECUDA, std::string("logits: ") + cudaGetErrorString(e));
  return Q35_OK;
}

// ---------------------------------------------------------------------------
// op-level entry points
// ---------------------------------------------------------------------------
static int op_status(cudaError_t e) { return e == cudaSuccess ? Q35_OK : Q35_ECUDA; }

int q35_op_qmv_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                  const uint16_t* x, const uint16_t* residual, uint16_t* y, int n, int k,
                  void* stream) {
  if (!w || !scales || !biases || !x || !y || n <= 0 || k <= 0 || k % 512 != 0 || k > 4096)
    return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  if (residual && residual != y) {
    cudaError_t e = cudaMemcpyAsync(y, residual, size_t(n) * 2, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return Q35_ECUDA;
  }
  QmvArgs a = {};
  a.seg[0] = {w, scales, biases, y, n};
  a.nseg = 1;
  a.K = k;
  a.units = n;
  int upc = (n + 147) / 148;
  upc = std::max(1, std::min(upc, qmv_max_rows(k)));
  a.units_per_cta = upc;
  a.pro = kProPlain;
  a.x = x;
  a.epi = residual ? kEpiResAdd : kEpiStore;
  a.res = y;
  return op_status(launch_qmv(a, st, false));
}

size_t q35_op_qgemm_workspace_bytes(uint32_t tokens, uint32_t n, uint32_t k) {
  if (tokens == 0 || tokens > 4096 || n == 0 || n > 524288 || k < 512 || k % 512 != 0 || k > 4096) return 0;
  return qgemm_workspace_bytes(int(n), int(k), int(tokens));
}

int q35_op_qgemm_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                    uint32_t tokens, uint32_t n, uint32_t k, const uint16_t* residual, uint16_t* y,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!w || !scales || !biases || !x || !y || !workspace || tokens < 1 || tokens > 4096 || n < 1 ||
      n > 524288 || k < 512 || k % 512 != 0 || k > 4096)
    return Q35_EINVAL;
  for (const void* p : {static_cast<const void*>(scales), static_cast<const void*>(biases)})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return Q35_EINVAL;
  for (const void* p : {static_cast<const void*>(w), static_cast<const void*>(x),
                        static_cast<const void*>(workspace)})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return Q35_EINVAL;
  if (workspace_bytes < qgemm_workspace_bytes(int(n), int(k), int(tokens))) return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  QGemmArgs a = {};
  a.nseg = 1;
  a.seg[0] = {w, scales, biases, y, residual, int(n), int(n)};
  a.x = x;
  a.K = int(k);
  a.T = int(tokens);
  return op_status(launch_qgemm(a, workspace, workspace_bytes, true, (cudaStream_t)stream, false));
}

int q35_op_embedding_q4(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        uint32_t token, int k, uint16_t* out, void* stream) {
  if (!w || !scales || !biases || !out || k <= 0 || k % 64 != 0) return Q35_EINVAL;
  return op_status(launch_embedding(w, scales, biases, token, k, out, (cudaStream_t)stream));
}

int q35_op_rms_norm(const uint16_t* x, const uint16_t* gain, uint16_t* out, void* stream) {
  if (!x || !gain || !out) return Q35_EINVAL;
  return op_status(launch_rms1024(x, gain, out, (cudaStream_t)stream));
}

static size_t ctl_bytes() { return (sizeof(Ctl) + 255) & ~size_t(255); }

size_t q35_op_gdn_workspace_bytes(void) { return ctl_bytes() + kGdnConv * 2 + 2048 * 2; }

int q35_op_gdn_step(const uint16_t* raw_qkv, const uint16_t* z, const uint16_t* a_raw,
                    const uint16_t* b_raw, uint16_t* history, const uint16_t* conv_w,
                    const float* a_log, const uint16_t* dt_bias, float* state,
                    const uint16_t* norm_w, const uint32_t* ow, const uint16_t* os,
                    const uint16_t* ob, const uint16_t* residual, uint16_t* out, void* workspace,
                    void* stream) {
  if (!raw_qkv || !z || !a_raw || !b_raw || !history || !conv_w || !a_log || !dt_bias || !state ||
      !norm_w || !ow || !os || !ob || !out || !workspace)
    return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  Ctl* ctl = (Ctl*)ws;
  uint16_t* conv = (uint16_t*)(ws + ctl_bytes());
  uint16_t* y = conv + kGdnConv;
  cudaError_t e = cudaMemsetAsync(ctl, 0, sizeof(Ctl), st);
  if (e == cudaSuccess) e = launch_gdn_conv(raw_qkv, history, conv_w, conv, st);
  RecurArgs r = {};
  r.conv = conv;
  r.a_raw = a_raw;
  r.b_raw = b_raw;
  r.a_log = a_log;
  r.dt_bias = dt_bias;
  r.state = state;
  r.y = y;
  r.ctl = ctl;
  if (e == cudaSuccess) e = launch_recur(r, st, false);
  if (e == cudaSuccess && residual && residual != out)
    e = cudaMemcpyAsync(out, residual, 1024 * 2, cudaMemcpyDeviceToDevice, st);
  QmvArgs o = {};
  o.seg[0] = {ow, os, ob, out, 1024};
  o.nseg = 1;
  o.K = 2048;
  o.units = 1024;
  o.units_per_cta = 7;
  o.pro = kProNormGate;
  o.gy = y;
  o.gz = z;
  o.gw = norm_w;
  o.epi = residual ? kEpiResAdd : kEpiStore;
  o.res = out;
  o.ctl = ctl;
  if (e == cudaSuccess) e = launch_qmv(o, st, false);
  return op_status(e);
}

int q35_op_status(const void* workspace, uint32_t kind, uint32_t* site, void* stream) {
  if (kind > Q35_OPWS_QGEMM) return Q35_EINVAL;
  const uint8_t* base = static_cast<const uint8_t*>(workspace);
  if (!base) {
    if (kind != Q35_OPWS_CTL) return Q35_EINVAL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q35_ECUDA;
    base = noalloc_scratch(dev);
    if (!base) return Q35_EINVAL;  // no allocation-free call on this device yet
  }
  const uint8_t* word = base + (kind == Q35_OPWS_QGEMM ? qgemm_err_offset() : offsetof(Ctl, err));
  uint32_t v = 0;
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaMemcpy(&v, word, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return Q35_ECUDA;
  if (site) *site = v;
  return v ? Q35_ETIMEOUT : Q35_OK;
}

size_t q35_op_attn_workspace_bytes(void) {
  return ctl_bytes() + size_t(kKvHeads) * kAttnChains * 4 * kHeadDim * 4 +
         size_t(kKvHeads) * kAttnChains * 4 * 2 * 4;
}

int q35_op_attn_decode(const uint16_t* q_raw, const uint16_t* k_raw, const uint16_t* v_raw,
                       const uint16_t* q_gain, const uint16_t* k_gain, uint16_t* kcache,
                       uint16_t* vcache, uint32_t capacity, uint32_t pos, uint16_t* gated,
                       void* workspace, void* stream) {
  if (!q_raw || !k_raw || !v_raw || !q_gain || !k_gain || !kcache || !vcache || !gated ||
      !workspace || capacity == 0 || capacity % kAttnChains != 0 || pos >= capacity)
    return Q35_EINVAL;
  for (const void* p : {(const void*)q_raw, (const void*)k_raw, (const void*)v_raw, (const void*)q_gain,
                        (const void*)k_gain, (const void*)kcache, (const void*)vcache})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  Ctl* ctl = (Ctl*)ws;
  float* po = (float*)(ws + ctl_bytes());
  float* pml = po + size_t(kKvHeads) * kAttnChains * 4 * kHeadDim;
  cudaError_t e = launch_ctl_position(ctl, pos, st);
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
  return op_status(e);
}

// Scratch of the prompt-chunk ops for `tokens` rows (rounded up to 32) and
// the attention partials of a cache of `capacity` positions, after a control
// block.
namespace {
struct PromptOpWs {
  Ctl* ctl;
  uint16_t *conv, *y, *qn;
  float *zs, *kq, *gb, *vv, *rope, *opart, *oml, *omax;
  size_t total;
};
PromptOpWs prompt_op_ws(uint8_t* base, uint32_t tokens, uint32_t capacity) {
  const size_t N = (size_t(tokens) + 31) / 32 * 32;
  const size_t items = prompt_attn_items_max(int(N), capacity);
  PromptOpWs w = {};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  w.ctl = (Ctl*)take(ctl_bytes());
  w.conv = (uint16_t*)take(N * kGdnConv * 2);
  w.y = (uint16_t*)take(N * 2048 * 2);
  w.qn = (uint16_t*)take(8 * N * 256 * 2);
  w.zs = (float*)take(N * 2048 * 4);
  w.kq = (float*)take(16 * N * 256 * 4);
  w.gb = (float*)take(16 * N * 2 * 4);
  w.vv = (float*)take(16 * 8 * N * 16 * 4);
  w.rope = (float*)take(N * 64 * 4);
  w.opart = (float*)take(items * 128 * 256 * 4);
  w.oml = (float*)take(items * 128 * 2 * 4);
  w.omax = (float*)take(items * 128 * 4);
  w.total = off;
  return w;
}
bool aligned16(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return false;
  return true;
}
}  // namespace

size_t q35_op_prompt_workspace_bytes(uint32_t tokens, uint32_t capacity) {
  if (tokens == 0 || tokens > uint32_t(kPromptChunk) || capacity % kAttnChains != 0) return 0;
  return prompt_op_ws(nullptr, tokens, capacity).total;
}

int q35_op_prompt_gdn(const uint16_t* raw_qkv, const uint16_t* z, const uint16_t* ab, uint16_t* history,
                      const uint16_t* conv_w, const float* a_log, const uint16_t* dt_bias, float* state,
                      const uint16_t* norm_w, uint32_t tokens, uint16_t* gated, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!raw_qkv || !z || !ab || !history || !conv_w || !a_log || !dt_bias || !state || !norm_w || !gated ||
      !workspace || tokens == 0 || tokens > uint32_t(kPromptChunk) ||
      workspace_bytes < q35_op_prompt_workspace_bytes(tokens, 0))
    return Q35_EINVAL;
  if (!aligned16({raw_qkv, z, state, gated, workspace, norm_w})) return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const PromptOpWs w = prompt_op_ws((uint8_t*)workspace, tokens, 0);
  PromptArgs pa = {};
  pa.T = int(tokens);
  pa.tmax = int((tokens + 31) / 32 * 32);
  pa.ctl = w.ctl;
  pa.raw = raw_qkv;
  pa.hist = history;
  pa.convw = conv_w;
  pa.conv = w.conv;
  pa.ab = ab;
  pa.z = z;
  pa.zs = w.zs;
  pa.a_log = a_log;
  pa.dt_bias = dt_bias;
  pa.kq = w.kq;
  pa.gb = w.gb;
  pa.vv = w.vv;
  pa.state = state;
  pa.y = w.y;
  cudaError_t e = launch_ctl_position(w.ctl, 0, st);
  if (e == cudaSuccess) e = launch_prompt_conv(pa, st, false);
  if (e == cudaSuccess) e = launch_prompt_gdn_prep(pa, st, true);
  if (e == cudaSuccess) e = launch_prompt_recur(pa, st, true);
  TokArgs g = {};
  g.n = int(tokens);
  g.y = w.y;
  g.zs = w.zs;
  g.gw = norm_w;
  g.gated = gated;
  if (e == cudaSuccess) e = launch_tok_normgate(g, st, true);
  return op_status(e);
}

int q35_op_prompt_attention(const uint16_t* q_raw, const uint16_t* k_raw, const uint16_t* v_raw,
                            const uint16_t* q_gain, const uint16_t* k_gain, uint16_t* kcache, uint16_t* vcache,
                            uint32_t capacity, uint32_t p0, uint32_t tokens, uint16_t* gated, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!q_raw || !k_raw || !v_raw || !q_gain || !k_gain || !kcache || !vcache || !gated || !workspace ||
      tokens == 0 || tokens > uint32_t(kPromptChunk) || capacity == 0 || capacity % kAttnChains != 0 ||
      uint64_t(p0) + tokens > capacity || workspace_bytes < q35_op_prompt_workspace_bytes(tokens, capacity))
    return Q35_EINVAL;
  if (!aligned16({q_raw, k_raw, v_raw, q_gain, k_gain, kcache, vcache, gated, workspace})) return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  const PromptOpWs w = prompt_op_ws((uint8_t*)workspace, tokens, capacity);
  PromptArgs pa = {};
  pa.T = int(tokens);
  pa.p0 = p0;
  pa.tmax = int((tokens + 31) / 32 * 32);
  pa.ctl = w.ctl;
  pa.q_raw = q_raw;
  pa.k_raw = k_raw;
  pa.v_raw = v_raw;
  pa.q_gain = q_gain;
  pa.k_gain = k_gain;
  pa.rope = w.rope;
  pa.qn = w.qn;
  pa.kcache = kcache;
  pa.vcache = vcache;
  pa.capacity = capacity;
  pa.opart = w.opart;
  pa.oml = w.oml;
  pa.omax = w.omax;
  pa.gated = gated;
  prompt_attn_plan(pa);
  cudaError_t e = launch_ctl_position(w.ctl, p0, st);
  if (e == cudaSuccess) e = launch_prompt_rope(p0, int(tokens), w.rope, st, false);
  if (e == cudaSuccess) e = launch_prompt_attn_prep(pa, st, true);
  if (e == cudaSuccess) e = launch_prompt_attn(pa, st, true);
  return op_status(e);
}

size_t q35_op_head_workspace_bytes(void) { return ctl_bytes() + size_t(kHeadCtas) * 2 * 4; }

int q35_op_head_argmax(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                       const uint16_t* x, const uint16_t* gain, uint16_t* logits,
                       uint32_t* token, uint16_t* lse, void* workspace, void* stream) {
  if (!w || !scales || !biases || !x || !logits || !token || !workspace) return Q35_EINVAL;
  if (ensure_kernels_init() != cudaSuccess) return Q35_ECUDA;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  Ctl* ctl = (Ctl*)ws;
  float* part = (float*)(ws + ctl_bytes());
  cudaError_t e = launch_ctl_position(ctl, 0, st);
  HeadArgs hd = {};
  hd.w = w;
  hd.s = scales;
  hd.b = biases;
  hd.x = x;
  hd.gain = gain;
  hd.logits = logits;
  hd.part = part;
  hd.seq = nullptr;
  hd.out_tokens = token;
  hd.seq_len = 0;
  hd.out_len = 1;
  hd.lse_out = lse;
  hd.ctl = ctl;
  if (e == cudaSuccess) e = launch_head(hd, st, false);
  return op_status(e);
}

int q35_op_greedy(const uint16_t* logits, uint32_t* token, uint16_t* lse, void* workspace,
                  void* stream) {
  if (!logits || !token || !workspace) return Q35_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  Ctl* ctl = (Ctl*)ws;
  float* part = (float*)(ws + ctl_bytes());
  cudaError_t e = launch_ctl_position(ctl, 0, st);
  HeadArgs hd = {};
  hd.logits = const_cast<uint16_t*>(logits);
  hd.part = part;
  hd.out_tokens = token;
  hd.out_len = 1;
  hd.lse_out = lse;
  hd.ctl = ctl;
  if (e == cudaSuccess) e = launch_greedy(hd, st);
  return op_status(e);
}

}  // extern "C"
