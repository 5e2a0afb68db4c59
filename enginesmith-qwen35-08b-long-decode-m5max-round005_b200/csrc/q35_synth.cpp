// Seeded random-init model writer (the checkpoint itself is not available
// offline). Produces config.json and model.safetensors with the 694
// language_model.model.* tensors that weights.rs/model.rs expect:
//   linears      Q4 affine, group 64, quantised from N(0, 0.02)
//   norm gains   bf16(1 + N(0, 0.02))
//   conv1d       bf16 N(0, 0.3)        dt_bias  bf16 U(-1, 1)
//   A_log        f32 U(-1, 1)
// Values depend only on (seed, tensor name, element index), through a
// splitmix64 counter generator, so any subset can be regenerated.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <vector>

#include "q35.h"

namespace {

uint64_t mix(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
uint64_t name_key(uint64_t seed, const std::string& name) {
  uint64_t h = 0xcbf29ce484222325ull ^ seed;
  for (unsigned char c : name) h = (h ^ c) * 0x100000001b3ull;
  return mix(h);
}
// uniform in [0,1) from 53 bits
double uni(uint64_t key, uint64_t i) { return double(mix(key + i * 0x632be59bd9b4e019ull) >> 11) * (1.0 / 9007199254740992.0); }
float normal(uint64_t key, uint64_t i) {
  const uint64_t p = i >> 1;
  double u1 = uni(key, 2 * p), u2 = uni(key, 2 * p + 1);
  if (u1 < 1e-300) u1 = 1e-300;
  const double r = std::sqrt(-2.0 * std::log(u1)), t = 6.283185307179586 * u2;
  return float((i & 1) ? r * std::sin(t) : r * std::cos(t));
}
uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
float bf2f(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

struct Spec {
  std::string name, dtype;
  std::vector<size_t> shape;
  int kind;  // 0 q4 codes, 1 q4 scales, 2 q4 biases, 3 gain, 4 conv, 5 dt, 6 alog
  std::string base;  // linear base name for q4 parts
  size_t n = 0, k = 0;
};

void parallel(size_t n, const std::function<void(size_t, size_t)>& fn);

void gen_q4(uint64_t key, size_t n, size_t k, uint32_t* codes, uint16_t* sc, uint16_t* bi) {
  const size_t groups = k / 64;
  parallel(n, [&](size_t r0, size_t r1) {
    std::vector<float> w(64);
    for (size_t r = r0; r < r1; ++r)
      for (size_t g = 0; g < groups; ++g) {
        float lo = 1e30f, hi = -1e30f;
        for (size_t j = 0; j < 64; ++j) {
          w[j] = 0.02f * normal(key, r * k + g * 64 + j);
          lo = std::min(lo, w[j]);
          hi = std::max(hi, w[j]);
        }
        float scale = bf2f(f2bf((hi - lo) / 15.0f));
        if (scale <= 0.0f) scale = 1e-8f;
        const float bias = bf2f(f2bf(lo));
        sc[r * groups + g] = f2bf(scale);
        bi[r * groups + g] = f2bf(bias);
        for (size_t j = 0; j < 64; j += 8) {
          uint32_t word = 0;
          for (size_t t = 0; t < 8; ++t) {
            long q = std::lround((w[j + t] - bias) / scale);
            q = std::max(0L, std::min(15L, q));
            word |= uint32_t(q) << (4 * t);
          }
          codes[(r * k + g * 64 + j) / 8] = word;
        }
      }
  });
}

void parallel(size_t n, const std::function<void(size_t, size_t)>& fn) {
  unsigned t = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  if (n < 64) t = 1;
  std::vector<std::thread> th;
  size_t chunk = (n + t - 1) / t;
  for (unsigned i = 0; i < t; ++i) {
    size_t a = i * chunk, b = std::min(n, a + chunk);
    if (a < b) th.emplace_back(fn, a, b);
  }
  for (auto& x : th) x.join();
}

void add_linear(std::vector<Spec>& v, const std::string& base, size_t n, size_t k) {
  v.push_back({base + ".weight", "U32", {n, k / 8}, 0, base, n, k});
  v.push_back({base + ".scales", "BF16", {n, k / 64}, 1, base, n, k});
  v.push_back({base + ".biases", "BF16", {n, k / 64}, 2, base, n, k});
}

std::vector<Spec> model_specs() {
  std::vector<Spec> v;
  add_linear(v, "embed_tokens", 248320, 1024);
  v.push_back({"norm.weight", "BF16", {1024}, 3});
  for (int l = 0; l < 24; ++l) {
    const std::string p = "layers." + std::to_string(l);
    v.push_back({p + ".input_layernorm.weight", "BF16", {1024}, 3});
    v.push_back({p + ".post_attention_layernorm.weight", "BF16", {1024}, 3});
    add_linear(v, p + ".mlp.gate_proj", 3584, 1024);
    add_linear(v, p + ".mlp.up_proj", 3584, 1024);
    add_linear(v, p + ".mlp.down_proj", 1024, 3584);
    if (l % 4 == 3) {
      const std::string a = p + ".self_attn";
      add_linear(v, a + ".q_proj", 4096, 1024);
      add_linear(v, a + ".k_proj", 512, 1024);
      add_linear(v, a + ".v_proj", 512, 1024);
      add_linear(v, a + ".o_proj", 1024, 2048);
      v.push_back({a + ".q_norm.weight", "BF16", {256}, 3});
      v.push_back({a + ".k_norm.weight", "BF16", {256}, 3});
    } else {
      const std::string a = p + ".linear_attn";
      add_linear(v, a + ".in_proj_qkv", 6144, 1024);
      add_linear(v, a + ".in_proj_z", 2048, 1024);
      add_linear(v, a + ".in_proj_a", 16, 1024);
      add_linear(v, a + ".in_proj_b", 16, 1024);
      add_linear(v, a + ".out_proj", 1024, 2048);
      v.push_back({a + ".conv1d.weight", "BF16", {6144, 4, 1}, 4});
      v.push_back({a + ".norm.weight", "BF16", {128}, 3});
      v.push_back({a + ".dt_bias", "BF16", {16}, 5});
      v.push_back({a + ".A_log", "F32", {16}, 6});
    }
  }
  return v;
}

size_t nbytes(const Spec& s) {
  size_t c = 1;
  for (size_t d : s.shape) c *= d;
  return c * (s.dtype == "BF16" ? 2 : 4);
}

}  // namespace

extern "C" int q35_write_synthetic_model(const char* dir, uint64_t seed, char* err, size_t err_len) {
  auto fail = [&](const std::string& m) {
    if (err && err_len) std::snprintf(err, err_len, "%s", m.c_str());
    return Q35_EIO;
  };
  if (!dir) return fail("no directory");
  ::mkdir(dir, 0755);
  std::vector<Spec> specs = model_specs();
  std::sort(specs.begin(), specs.end(), [](const Spec& a, const Spec& b) { return a.name < b.name; });
  // header
  std::string h = "{\"__metadata__\":{\"format\":\"mlx\"}";
  size_t off = 0;
  std::vector<size_t> offs;
  for (auto& s : specs) {
    const size_t b = nbytes(s);
    offs.push_back(off);
    h += ",\"language_model.model." + s.name + "\":{\"dtype\":\"" + s.dtype + "\",\"shape\":[";
    for (size_t i = 0; i < s.shape.size(); ++i) h += (i ? "," : "") + std::to_string(s.shape[i]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + b) + "]}";
    off += b;
  }
  h += "}";
  while ((h.size() + 8) % 16) h += ' ';
  std::vector<uint8_t> data(off);
  // q4 triples are generated together from the linear's key
  for (size_t i = 0; i < specs.size(); ++i) {
    const Spec& s = specs[i];
    uint8_t* dst = data.data() + offs[i];
    const size_t count = nbytes(s) / (s.dtype == "BF16" ? 2 : 4);
    const uint64_t key = name_key(seed, s.kind <= 2 ? s.base : s.name);
    if (s.kind == 0) {
      size_t si = 0, bi = 0;
      for (size_t j = 0; j < specs.size(); ++j) {
        if (specs[j].base == s.base && specs[j].kind == 1) si = j;
        if (specs[j].base == s.base && specs[j].kind == 2) bi = j;
      }
      gen_q4(key, s.n, s.k, reinterpret_cast<uint32_t*>(dst),
             reinterpret_cast<uint16_t*>(data.data() + offs[si]),
             reinterpret_cast<uint16_t*>(data.data() + offs[bi]));
    } else if (s.kind == 3 || s.kind == 4 || s.kind == 5) {
      uint16_t* o = reinterpret_cast<uint16_t*>(dst);
      for (size_t j = 0; j < count; ++j) {
        float v = s.kind == 3 ? 1.0f + 0.02f * normal(key, j)
                  : s.kind == 4 ? 0.3f * normal(key, j)
                                : float(2.0 * uni(key, j) - 1.0);
        o[j] = f2bf(v);
      }
    } else if (s.kind == 6) {
      float* o = reinterpret_cast<float*>(dst);
      for (size_t j = 0; j < count; ++j) o[j] = float(2.0 * uni(key, j) - 1.0);
    }
  }
  const std::string path = std::string(dir) + "/model.safetensors";
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return fail("cannot write " + path);
  const uint64_t hn = h.size();
  bool ok = std::fwrite(&hn, 8, 1, f) == 1 && std::fwrite(h.data(), 1, h.size(), f) == h.size() &&
            std::fwrite(data.data(), 1, data.size(), f) == data.size();
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) return fail("write failed: " + path);
  const std::string cfg =
      "{\"model_type\":\"qwen3_5\",\"architectures\":[\"Qwen3_5ForConditionalGeneration\"],"
      "\"quantization\":{\"group_size\":64,\"bits\":4,\"mode\":\"affine\"},"
      "\"text_config\":{\"hidden_size\":1024,\"num_hidden_layers\":24,\"vocab_size\":248320,"
      "\"intermediate_size\":3584,\"num_attention_heads\":8,\"num_key_value_heads\":2,"
      "\"head_dim\":256,\"linear_num_key_heads\":16,\"linear_num_value_heads\":16,"
      "\"linear_key_head_dim\":128,\"linear_value_head_dim\":128,\"linear_conv_kernel_dim\":4,"
      "\"full_attention_interval\":4,\"rms_norm_eps\":1e-06,\"rope_theta\":10000000,"
      "\"partial_rotary_factor\":0.25,\"tie_word_embeddings\":true},"
      "\"synthetic\":{\"seed\":" + std::to_string(seed) + "}}\n";
  f = std::fopen((std::string(dir) + "/config.json").c_str(), "wb");
  if (!f) return fail("cannot write config.json");
  ok = std::fwrite(cfg.data(), 1, cfg.size(), f) == cfg.size();
  ok = (std::fclose(f) == 0) && ok;
  return ok ? Q35_OK : fail("write failed: config.json");
}
