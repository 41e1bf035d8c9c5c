// gguf.cu — the decoder's weights straight from a GGUF file.
//
// wg_model_create_from_gguf replaces gguf.Open + model.NewDecoder
// (internal/gguf/gguf.go:52-134, internal/model/decoder.go:97-303) for the
// decoder half of a whisper.go model file: the file is mapped read-only, the
// header, metadata and tensor table are parsed in place (GGUF v2/v3, the
// value types of internal/gguf/metadata.go:10-24), every decoder tensor is
// found under its whisper.cpp name or its Hugging Face name (the table of
// internal/model/compat.go:31-148), and the quantised blocks are handed to
// wg_model_create as pointers into the mapping, so they go from the page
// cache to the device without a host copy (the repack into the device layout
// happens on upload). Only fp32 vectors stored as F16, and dense matrices
// stored transposed, are converted on the host.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cerrno>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "kernels.cuh"

namespace wg {
namespace {

constexpr uint32_t GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7,
                   GT_STR = 8, GT_ARR = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12;

struct Tensor {
  std::vector<uint64_t> shape;
  uint32_t dtype = 0;
  uint64_t offset = 0;
};

struct Gguf {
  const uint8_t* base = nullptr;
  size_t size = 0;
  std::map<std::string, uint32_t> meta_u32;  // metadata of type uint32 (MetaUint32 reads only those)
  std::map<std::string, Tensor> tensors;
  uint64_t data_start = 0;
  std::string err;

  // bounded little-endian reader over the mapping
  size_t pos = 0;
  bool need(size_t n) {
    if (pos + n > size || pos + n < pos) {
      err = "gguf: truncated file";
      return false;
    }
    return true;
  }
  template <typename T>
  bool rd(T* v) {
    if (!need(sizeof(T))) return false;
    memcpy(v, base + pos, sizeof(T));
    pos += sizeof(T);
    return true;
  }
  bool str(std::string* s) {
    uint64_t n = 0;
    if (!rd(&n) || !need(n)) return false;
    if (s) s->assign(reinterpret_cast<const char*>(base + pos), n);
    pos += n;
    return true;
  }
  static int scalar_bytes(uint32_t t) {
    switch (t) {
      case GT_U8: case GT_I8: case GT_BOOL: return 1;
      case GT_U16: case GT_I16: return 2;
      case GT_U32: case GT_I32: case GT_F32: return 4;
      case GT_U64: case GT_I64: case GT_F64: return 8;
      default: return 0;
    }
  }
  bool skip_value(uint32_t t, int depth = 0) {
    if (t == GT_STR) return str(nullptr);
    if (t == GT_ARR) {
      uint32_t et = 0;
      uint64_t n = 0;
      if (depth > 4 || !rd(&et) || !rd(&n)) return depth > 4 ? (err = "gguf: nested arrays", false) : false;
      if (const int b = scalar_bytes(et)) {
        if (n > size / (uint64_t)b || !need((size_t)n * b)) return false;
        pos += (size_t)n * b;
        return true;
      }
      for (uint64_t i = 0; i < n; i++)
        if (!skip_value(et, depth + 1)) return false;
      return true;
    }
    const int b = scalar_bytes(t);
    if (!b) {
      err = "gguf: unknown value type " + std::to_string(t);
      return false;
    }
    if (!need(b)) return false;
    pos += b;
    return true;
  }

  // gguf.go:69-134
  bool parse() {
    if (size < 4 || memcmp(base, "GGUF", 4) != 0) {
      err = "gguf: invalid magic";
      return false;
    }
    pos = 4;
    uint32_t version = 0;
    uint64_t n_tensors = 0, n_meta = 0;
    if (!rd(&version)) return false;
    if (version != 2 && version != 3) {
      err = "gguf: unsupported version: " + std::to_string(version);
      return false;
    }
    if (!rd(&n_tensors) || !rd(&n_meta)) return false;
    for (uint64_t i = 0; i < n_meta; i++) {
      std::string key;
      uint32_t t = 0;
      if (!str(&key) || !rd(&t)) return false;
      if (t == GT_U32) {
        uint32_t v = 0;
        if (!rd(&v)) return false;
        meta_u32[key] = v;
      } else if (!skip_value(t)) {
        return false;
      }
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
      std::string name;
      uint32_t nd = 0;
      Tensor td;
      if (!str(&name) || !rd(&nd)) return false;
      if (nd > 8) {
        err = "gguf: tensor " + name + " has " + std::to_string(nd) + " dimensions";
        return false;
      }
      td.shape.resize(nd);
      for (uint32_t k = 0; k < nd; k++)
        if (!rd(&td.shape[k])) return false;
      if (!rd(&td.dtype) || !rd(&td.offset)) return false;
      tensors[name] = td;
    }
    uint64_t align = 32;
    auto a = meta_u32.find("general.alignment");
    if (a != meta_u32.end() && a->second > 0) align = a->second;
    data_start = (pos + align - 1) / align * align;
    return true;
  }

  // bytes of n elements of dtype (tensor.go:61-88); 0 if unsupported
  static uint64_t raw_bytes(uint32_t dtype, uint64_t n) {
    const uint64_t nb = (n + 31) / 32;
    switch (dtype) {
      case WG_QTYPE_F32: return n * 4;
      case WG_QTYPE_F16: return n * 2;
      case WG_QTYPE_Q4_0: return nb * 18;
      case WG_QTYPE_Q4_1: return nb * 20;
      case WG_QTYPE_Q5_0: return nb * 22;
      case WG_QTYPE_Q5_1: return nb * 24;
      case WG_QTYPE_Q8_0: return nb * 34;
      default: return 0;
    }
  }
  // The tensor's bytes inside the mapping, checked against the file size.
  const uint8_t* data(const Tensor& t, uint64_t* elems) {
    uint64_t n = 1;
    for (uint64_t d : t.shape) n *= d;
    const uint64_t nb = raw_bytes(t.dtype, n);
    if (!nb || data_start + t.offset + nb > size || data_start + t.offset < data_start) return nullptr;
    if (elems) *elems = n;
    return base + data_start + t.offset;
  }
};

// compat.go:31-148, the decoder half: whisper.cpp name -> Hugging Face name.
std::string hf_name(const std::string& name) {
  static const std::map<std::string, std::string> simple = {
      {"decoder.token_embedding.weight", "model.decoder.embed_tokens.weight"},
      {"decoder.positional_embedding", "model.decoder.embed_positions.weight"},
      {"decoder.ln.weight", "model.decoder.layer_norm.weight"},
      {"decoder.ln.bias", "model.decoder.layer_norm.bias"},
  };
  auto it = simple.find(name);
  if (it != simple.end()) return it->second;
  static const std::string pre = "decoder.blocks.";
  if (name.compare(0, pre.size(), pre) != 0) return "";
  size_t i = pre.size(), j = i;
  while (j < name.size() && isdigit((unsigned char)name[j])) j++;
  if (j == i || j >= name.size() || name[j] != '.') return "";
  const std::string idx = name.substr(i, j - i), suffix = name.substr(j + 1);
  static const std::map<std::string, std::string> blk = {
      {"self_attn_ln.weight", "self_attn_layer_norm.weight"}, {"self_attn_ln.bias", "self_attn_layer_norm.bias"},
      {"self_attn.query.weight", "self_attn.q_proj.weight"},   {"self_attn.query.bias", "self_attn.q_proj.bias"},
      {"self_attn.key.weight", "self_attn.k_proj.weight"},     {"self_attn.value.weight", "self_attn.v_proj.weight"},
      {"self_attn.value.bias", "self_attn.v_proj.bias"},       {"self_attn.out.weight", "self_attn.out_proj.weight"},
      {"self_attn.out.bias", "self_attn.out_proj.bias"},       {"cross_attn_ln.weight", "encoder_attn_layer_norm.weight"},
      {"cross_attn_ln.bias", "encoder_attn_layer_norm.bias"},  {"cross_attn.query.weight", "encoder_attn.q_proj.weight"},
      {"cross_attn.query.bias", "encoder_attn.q_proj.bias"},   {"cross_attn.key.weight", "encoder_attn.k_proj.weight"},
      {"cross_attn.value.weight", "encoder_attn.v_proj.weight"}, {"cross_attn.value.bias", "encoder_attn.v_proj.bias"},
      {"cross_attn.out.weight", "encoder_attn.out_proj.weight"}, {"cross_attn.out.bias", "encoder_attn.out_proj.bias"},
      {"mlp_ln.weight", "final_layer_norm.weight"},            {"mlp_ln.bias", "final_layer_norm.bias"},
      {"mlp.0.weight", "fc1.weight"},                          {"mlp.0.bias", "fc1.bias"},
      {"mlp.2.weight", "fc2.weight"},                          {"mlp.2.bias", "fc2.bias"},
  };
  auto b = blk.find(suffix);
  return b == blk.end() ? "" : "model.decoder.layers." + idx + "." + b->second;
}

// The loader's state: the mapping, the tensors found, and the host buffers
// of the converted ones (all released after the upload).
struct Loader {
  Gguf g;
  std::vector<std::unique_ptr<std::vector<float>>> keep;
  std::string err;

  const Tensor* find(const std::string& name, std::string* resolved) {  // compat.go:15-29
    auto it = g.tensors.find(name);
    if (it != g.tensors.end()) {
      if (resolved) *resolved = name;
      return &it->second;
    }
    const std::string alt = hf_name(name);
    if (alt.empty()) return nullptr;
    it = g.tensors.find(alt);
    if (it == g.tensors.end()) return nullptr;
    if (resolved) *resolved = alt;
    return &it->second;
  }

  float* host(size_t n) {
    keep.emplace_back(new std::vector<float>(n));
    return keep.back()->data();
  }
  static float f16(uint16_t h) {  // IEEE binary16 -> float32 (exact), gguf/dequant.go:15-44
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t bits;
    if (e == 0) {
      if (m == 0) bits = s;
      else {
        int k = 0;
        uint32_t mm = m;
        while (!(mm & 0x400)) { mm <<= 1; k++; }
        bits = s | (uint32_t)(113 - k) << 23 | (mm & 0x3FF) << 13;
      }
    } else if (e == 31) {
      bits = s | 0x7F800000u | m << 13;
    } else {
      bits = s | (e + 112) << 23 | m << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
  }

  // An fp32 vector of n values (F32 in place; F16 converted).
  const float* vec(const std::string& name, uint64_t n) {
    std::string r;
    const Tensor* t = find(name, &r);
    uint64_t elems = 0;
    const uint8_t* p = t ? g.data(*t, &elems) : nullptr;
    if (!t) { err = "model: load tensor \"" + name + "\": not found"; return nullptr; }
    if (!p || elems != n || (t->dtype != WG_QTYPE_F32 && t->dtype != WG_QTYPE_F16)) {
      err = "model: load tensor \"" + name + "\" (resolved \"" + r + "\"): expected " + std::to_string(n) +
            " F32/F16 values";
      return nullptr;
    }
    if (t->dtype == WG_QTYPE_F32 && (reinterpret_cast<uintptr_t>(p) & 3) == 0) return reinterpret_cast<const float*>(p);
    float* o = host(n);
    for (uint64_t i = 0; i < n; i++) {
      if (t->dtype == WG_QTYPE_F32) memcpy(&o[i], p + 4 * i, 4);
      else {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        o[i] = f16(h);
      }
    }
    return o;
  }

  // A [rows, cols] matrix (loadMatWeightAuto, compat.go:247-270): quantised
  // or dense as stored; a dense matrix stored [cols, rows] is transposed.
  bool mat(const std::string& name, int rows, int cols, wg_matrix* m) {
    std::string r;
    const Tensor* t = find(name, &r);
    if (!t) { err = "model: load tensor \"" + name + "\": not found"; return false; }
    uint64_t elems = 0;
    const uint8_t* p = g.data(*t, &elems);
    if (!p || t->shape.size() != 2) {
      err = "model: invalid " + name + " (resolved \"" + r + "\"): unsupported type or shape";
      return false;
    }
    const uint64_t s0 = t->shape[0], s1 = t->shape[1];
    if (s0 == (uint64_t)rows && s1 == (uint64_t)cols) {
      *m = wg_matrix{t->dtype, rows, cols, p};
      return true;
    }
    if (s0 == (uint64_t)cols && s1 == (uint64_t)rows && (t->dtype == WG_QTYPE_F32 || t->dtype == WG_QTYPE_F16)) {
      float* o = host((size_t)rows * cols);
      for (int i = 0; i < rows; i++)
        for (int j = 0; j < cols; j++) {
          const size_t src = (size_t)j * rows + i;
          if (t->dtype == WG_QTYPE_F32) memcpy(&o[(size_t)i * cols + j], p + 4 * src, 4);
          else {
            uint16_t h;
            memcpy(&h, p + 2 * src, 2);
            o[(size_t)i * cols + j] = f16(h);
          }
        }
      *m = wg_matrix{WG_QTYPE_F32, rows, cols, o};
      return true;
    }
    err = "model: unsupported " + name + " shape [" + std::to_string(s0) + " " + std::to_string(s1) + "]";
    return false;
  }

  uint32_t meta(const char* a, const char* b = nullptr) {  // getMetaAny, compat.go:163-170
    auto it = g.meta_u32.find(a);
    if (it != g.meta_u32.end()) return it->second;
    if (b && (it = g.meta_u32.find(b)) != g.meta_u32.end()) return it->second;
    return 0;
  }
  const Tensor* shape_of(const std::string& name) { return find(name, nullptr); }
};

}  // namespace
}  // namespace wg

using namespace wg;

extern "C" int wg_model_create_from_gguf(const char* path, const int* devices, int n_dev, wg_model** out) {
  if (!path || !out) { set_error("wg_model_create_from_gguf: null argument"); return WG_ERR_INVALID; }
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) { set_error("gguf: open: %s: %s", path, strerror(errno)); return WG_ERR_INVALID; }
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
    close(fd);
    set_error("gguf: open: %s: empty or unreadable", path);
    return WG_ERR_INVALID;
  }
  void* map = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) { set_error("gguf: mmap of %s failed: %s", path, strerror(errno)); return WG_ERR_INVALID; }
  madvise(map, (size_t)sb.st_size, MADV_SEQUENTIAL);
  std::unique_ptr<Loader> ld(new Loader());
  ld->g.base = static_cast<const uint8_t*>(map);
  ld->g.size = (size_t)sb.st_size;
  int rc = WG_OK;
  auto fail = [&](const std::string& why) {
    set_error("%s", why.c_str());
    rc = WG_ERR_INVALID;
  };
  if (!ld->g.parse()) fail(ld->g.err);
  // hyper-parameters, as NewDecoder infers them (decoder.go:101-170)
  int H = 0, L = 0, ctx = 0, d = 0, V = 0;
  if (rc == WG_OK) {
    H = (int)ld->meta("whisper.decoder.attention.head_count");
    L = (int)ld->meta("whisper.decoder.layer_count");
    ctx = (int)ld->meta("whisper.decoder.context_length");
    d = (int)ld->meta("whisper.decoder.embedding_length");
    V = (int)ld->meta("whisper.vocab.size", "whisper.n_vocab");
    if (L == 0)
      while (ld->shape_of("decoder.blocks." + std::to_string(L) + ".self_attn.query.weight")) L++;
    if (const Tensor* q = ld->shape_of("decoder.blocks.0.self_attn.query.weight"))
      if (q->shape.size() == 2 && q->shape[0] == q->shape[1] && q->shape[0] > 0) d = (int)q->shape[0];
    if (ctx == 0 || d == 0) {
      const Tensor* p = ld->shape_of("decoder.positional_embedding");
      if (!p || p->shape.size() != 2) fail("model: decoder: invalid positional embedding");
      else if (d > 0) ctx = (int)(p->shape[0] == (uint64_t)d && p->shape[1] != (uint64_t)d ? p->shape[1] : p->shape[0]);
      else { ctx = (int)p->shape[0]; d = (int)p->shape[1]; }
    }
    if (rc == WG_OK && V == 0) {
      const Tensor* t = ld->shape_of("decoder.token_embedding.weight");
      if (!t || t->shape.size() != 2) fail("model: decoder: invalid token embedding");
      else V = (int)(t->shape[1] == (uint64_t)d ? t->shape[0] : t->shape[1]);
    }
    if (rc == WG_OK && H == 0) {
      if (d % 64) fail("model: decoder: cannot infer head count from embedding length " + std::to_string(d));
      else H = d / 64;
    }
    if (rc == WG_OK && (L <= 0 || d <= 0 || V <= 0 || ctx <= 0)) fail("model: decoder: incomplete hyper-parameters");
  }
  wg_model_desc desc{};
  std::vector<wg_layer_desc> layers(L > 0 ? L : 0);
  if (rc == WG_OK) {
    desc.n_vocab = V; desc.n_state = d; desc.n_head = H; desc.n_layer = L; desc.n_text_ctx = ctx;
    desc.eot = 50256;  // decoder.go:173; SetVocabulary may change it (wg_model_set_eot)
    Loader& l = *ld;
    bool ok = l.mat("decoder.token_embedding.weight", V, d, &desc.token_embedding);
    // positional embedding [ctx, d] (transposed if stored [d, ctx], decoder.go:189-197)
    if (ok) {
      std::string r;
      const Tensor* t = l.find("decoder.positional_embedding", &r);
      if (t && t->shape.size() == 2 && t->shape[0] == (uint64_t)d && t->shape[1] == (uint64_t)ctx && d != ctx) {
        wg_matrix m{};
        ok = l.mat("decoder.positional_embedding", ctx, d, &m);
        desc.positional_embedding = static_cast<const float*>(m.data);
      } else {
        desc.positional_embedding = l.vec("decoder.positional_embedding", (uint64_t)ctx * d);
        ok = desc.positional_embedding != nullptr;
      }
    }
    ok = ok && (desc.ln_w = l.vec("decoder.ln.weight", d)) && (desc.ln_b = l.vec("decoder.ln.bias", d));
    for (int i = 0; ok && i < L; i++) {
      const std::string p = "decoder.blocks." + std::to_string(i) + ".";
      wg_layer_desc& b = layers[i];
      ok = (b.self_ln_w = l.vec(p + "self_attn_ln.weight", d)) && (b.self_ln_b = l.vec(p + "self_attn_ln.bias", d)) &&
           l.mat(p + "self_attn.query.weight", d, d, &b.self_q) && (b.self_q_b = l.vec(p + "self_attn.query.bias", d)) &&
           l.mat(p + "self_attn.key.weight", d, d, &b.self_k) && l.mat(p + "self_attn.value.weight", d, d, &b.self_v) &&
           (b.self_v_b = l.vec(p + "self_attn.value.bias", d)) && l.mat(p + "self_attn.out.weight", d, d, &b.self_o) &&
           (b.self_o_b = l.vec(p + "self_attn.out.bias", d)) && (b.cross_ln_w = l.vec(p + "cross_attn_ln.weight", d)) &&
           (b.cross_ln_b = l.vec(p + "cross_attn_ln.bias", d)) &&
           l.mat(p + "cross_attn.query.weight", d, d, &b.cross_q) &&
           (b.cross_q_b = l.vec(p + "cross_attn.query.bias", d)) &&
           l.mat(p + "cross_attn.key.weight", d, d, &b.cross_k) && l.mat(p + "cross_attn.value.weight", d, d, &b.cross_v) &&
           (b.cross_v_b = l.vec(p + "cross_attn.value.bias", d)) &&
           l.mat(p + "cross_attn.out.weight", d, d, &b.cross_o) && (b.cross_o_b = l.vec(p + "cross_attn.out.bias", d)) &&
           (b.mlp_ln_w = l.vec(p + "mlp_ln.weight", d)) && (b.mlp_ln_b = l.vec(p + "mlp_ln.bias", d)) &&
           l.mat(p + "mlp.0.weight", 4 * d, d, &b.mlp0) && (b.mlp0_b = l.vec(p + "mlp.0.bias", (uint64_t)4 * d)) &&
           l.mat(p + "mlp.2.weight", d, 4 * d, &b.mlp2) && (b.mlp2_b = l.vec(p + "mlp.2.bias", d));
    }
    if (!ok) fail(l.err.empty() ? std::string("model: decoder: a tensor is missing") : l.err);
    desc.layers = layers.data();
  }
  if (rc == WG_OK) rc = wg_model_create(&desc, devices, n_dev, out);  // copies what it needs
  munmap(map, (size_t)sb.st_size);
  return rc;
}
