// GGUF (v2, v3) reader: the model loader the reference's engine expects
// behind InferenceEngine.Load (src/SharpInfer.Core/Engine/InferenceEngine.cs:
// 48-49; its Models/ loader is not in the repository).  It memory-maps the
// file, parses the metadata key/value table and the tensor table, derives
// the si_model_config of a Llama-architecture model from the metadata, and
// hands each weight's raw GGUF block bytes to si_model_set_tensor -- the
// quantised blocks go to the device as they are, never expanded to f32.
//
// File layout (little endian):
//   "GGUF", u32 version, u64 tensor count, u64 key/value count
//   key/value: string key, u32 type, value (arrays: u32 item type, u64 count, items)
//   tensor info: string name, u32 n_dims, u64 dims[n_dims] (dims[0] fastest),
//                u32 ggml type, u64 offset from the start of the data section
//   data section at the first multiple of general.alignment (default 32)
// Strings are u64 length + bytes.  The ggml type ids are the values of the
// reference's QuantType enum (Quantization.cs:6-22).
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

enum : uint32_t {
  GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7, GT_STR = 8,
  GT_ARR = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};

struct KV {
  uint32_t type = 0;
  uint64_t off = 0;        // file offset of the value (arrays: of the first item)
  uint32_t item_type = 0;  // arrays
  uint64_t count = 0;      // arrays
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;  // from the data section
  uint64_t bytes = 0;
};

// Block size (elements) and bytes of the ggml types (0 bytes: unknown).
void type_block(uint32_t t, uint64_t* elems, uint64_t* bytes) {
  switch (t) {
    case 0: *elems = 1; *bytes = 4; return;      // F32
    case 1: *elems = 1; *bytes = 2; return;      // F16
    case 2: *elems = 32; *bytes = 18; return;    // Q4_0
    case 3: *elems = 32; *bytes = 20; return;    // Q4_1
    case 6: *elems = 32; *bytes = 22; return;    // Q5_0
    case 7: *elems = 32; *bytes = 24; return;    // Q5_1
    case 8: *elems = 32; *bytes = 34; return;    // Q8_0
    case 9: *elems = 32; *bytes = 36; return;    // Q8_1
    case 10: *elems = 256; *bytes = 84; return;  // Q2_K
    case 11: *elems = 256; *bytes = 110; return; // Q3_K
    case 12: *elems = 256; *bytes = 144; return; // Q4_K
    case 13: *elems = 256; *bytes = 176; return; // Q5_K
    case 14: *elems = 256; *bytes = 210; return; // Q6_K
    case 15: *elems = 256; *bytes = 292; return; // Q8_K
    case 30: *elems = 1; *bytes = 2; return;     // BF16
    default: *elems = 1; *bytes = 0; return;
  }
}

}  // namespace

struct si_gguf {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32, data_off = 0;
  std::map<std::string, KV> kv;
  std::vector<TensorInfo> tensors;
  std::map<std::string, size_t> by_name;
};

namespace {

struct Cursor {
  const si_gguf* g;
  uint64_t pos;
  bool ok = true;
  bool need(uint64_t n) {
    if (!ok || pos + n > g->size || pos + n < pos) ok = false;
    return ok;
  }
  template <typename T>
  T rd() {
    T v{};
    if (need(sizeof(T))) {
      memcpy(&v, g->map + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  std::string str() {
    const uint64_t n = rd<uint64_t>();
    if (n > (1u << 24) || !need(n)) {
      ok = false;
      return {};
    }
    std::string s((const char*)g->map + pos, (size_t)n);
    pos += n;
    return s;
  }
};

uint64_t scalar_size(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
  }
}

// Skip one value of type t at the cursor (recording nothing).
bool skip_value(Cursor& c, uint32_t t) {
  if (t == GT_STR) {
    c.str();
    return c.ok;
  }
  if (t == GT_ARR) {
    const uint32_t it = c.rd<uint32_t>();
    const uint64_t n = c.rd<uint64_t>();
    if (!c.ok) return false;
    if (it == GT_STR || it == GT_ARR) {
      for (uint64_t i = 0; i < n && c.ok; i++) skip_value(c, it);
      return c.ok;
    }
    const uint64_t sz = scalar_size(it);
    if (!sz || n > (1ull << 40) || !c.need(sz * n)) return c.ok = false;
    c.pos += sz * n;
    return true;
  }
  const uint64_t sz = scalar_size(t);
  if (!sz || !c.need(sz)) return c.ok = false;
  c.pos += sz;
  return true;
}

int parse(si_gguf* g) {
  Cursor c{g, 0};
  if (g->size < 24 || memcmp(g->map, "GGUF", 4) != 0) SI_FAIL(SI_ERR_INVALID, "gguf: not a GGUF file (magic)");
  c.pos = 4;
  g->version = c.rd<uint32_t>();
  if (g->version != 2 && g->version != 3) SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: version %u (2 and 3 are read)", g->version);
  const uint64_t nt = c.rd<uint64_t>(), nkv = c.rd<uint64_t>();
  if (nt > (1u << 24) || nkv > (1u << 24)) SI_FAIL(SI_ERR_INVALID, "gguf: implausible table sizes");
  for (uint64_t i = 0; i < nkv && c.ok; i++) {
    const std::string key = c.str();
    KV v;
    v.type = c.rd<uint32_t>();
    if (v.type == GT_ARR) {
      v.item_type = c.rd<uint32_t>();
      v.count = c.rd<uint64_t>();
      v.off = c.pos;
      c.pos -= 12;  // skip_value re-reads the array header
    } else {
      v.off = c.pos;
    }
    if (!skip_value(c, v.type)) break;
    g->kv[key] = v;
  }
  if (!c.ok) SI_FAIL(SI_ERR_INVALID, "gguf: truncated or malformed key/value table");
  auto it = g->kv.find("general.alignment");
  if (it != g->kv.end()) {
    uint32_t a = 0;
    if (it->second.type == GT_U32) memcpy(&a, g->map + it->second.off, 4);
    if (a == 0 || (a & (a - 1))) SI_FAIL(SI_ERR_INVALID, "gguf: alignment %u is not a power of two", a);
    g->alignment = a;
  }
  g->tensors.resize((size_t)nt);
  for (uint64_t i = 0; i < nt && c.ok; i++) {
    TensorInfo& t = g->tensors[(size_t)i];
    t.name = c.str();
    const uint32_t nd = c.rd<uint32_t>();
    if (nd == 0 || nd > 4) c.ok = false;
    for (uint32_t d = 0; d < nd && c.ok; d++) t.dims.push_back(c.rd<uint64_t>());
    t.type = c.rd<uint32_t>();
    t.offset = c.rd<uint64_t>();
    uint64_t be, bb, n = 1;
    type_block(t.type, &be, &bb);
    for (uint64_t d : t.dims) n *= d;
    t.bytes = bb ? n / be * bb : 0;
    if (bb && (t.dims[0] % be)) c.ok = false;
    g->by_name[t.name] = (size_t)i;
  }
  if (!c.ok) SI_FAIL(SI_ERR_INVALID, "gguf: truncated or malformed tensor table");
  g->data_off = (c.pos + g->alignment - 1) / g->alignment * g->alignment;
  for (const TensorInfo& t : g->tensors)
    if (t.bytes && (g->data_off + t.offset + t.bytes > g->size || t.offset % g->alignment))
      SI_FAIL(SI_ERR_INVALID, "gguf: tensor %s lies outside the file", t.name.c_str());
  return SI_OK;
}

const KV* find_kv(const si_gguf* g, const char* key) {
  auto it = g->kv.find(key);
  return it == g->kv.end() ? nullptr : &it->second;
}

bool kv_int(const si_gguf* g, const std::string& key, int64_t* out) {
  const KV* v = find_kv(g, key.c_str());
  if (!v) return false;
  const uint8_t* p = g->map + v->off;
  switch (v->type) {
    case GT_U8: *out = *p; return true;
    case GT_I8: *out = (int8_t)*p; return true;
    case GT_BOOL: *out = *p != 0; return true;
    case GT_U16: { uint16_t x; memcpy(&x, p, 2); *out = x; return true; }
    case GT_I16: { int16_t x; memcpy(&x, p, 2); *out = x; return true; }
    case GT_U32: { uint32_t x; memcpy(&x, p, 4); *out = x; return true; }
    case GT_I32: { int32_t x; memcpy(&x, p, 4); *out = x; return true; }
    case GT_U64: { uint64_t x; memcpy(&x, p, 8); *out = (int64_t)x; return true; }
    case GT_I64: { int64_t x; memcpy(&x, p, 8); *out = x; return true; }
    default: return false;
  }
}

bool kv_float(const si_gguf* g, const std::string& key, double* out) {
  const KV* v = find_kv(g, key.c_str());
  if (!v) return false;
  if (v->type == GT_F32) {
    float x;
    memcpy(&x, g->map + v->off, 4);
    *out = x;
    return true;
  }
  if (v->type == GT_F64) {
    memcpy(out, g->map + v->off, 8);
    return true;
  }
  int64_t i;
  if (kv_int(g, key, &i)) {
    *out = (double)i;
    return true;
  }
  return false;
}

bool kv_str(const si_gguf* g, const std::string& key, std::string* out) {
  const KV* v = find_kv(g, key.c_str());
  if (!v || v->type != GT_STR) return false;
  Cursor c{g, v->off};
  *out = c.str();
  return c.ok;
}

const TensorInfo* find_tensor(const si_gguf* g, const std::string& name) {
  auto it = g->by_name.find(name);
  return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}

// Tensor names of the llama layout and the si_tensor ids they fill.
const char* kLayerNames[9] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
                              "attn_norm", "ffn_norm"};

std::string layer_name(int l, int t) { return "blk." + std::to_string(l) + "." + kLayerNames[t] + ".weight"; }

bool supported_weight(uint32_t t) { return t == SI_Q4_K || t == SI_Q6_K || t == SI_Q8_0; }

}  // namespace

using namespace si;

extern "C" {

SI_EXPORT int si_gguf_open(const char* path, si_gguf** out) {
  clear_error();
  if (!path || !out) SI_FAIL(SI_ERR_INVALID, "si_gguf_open: NULL argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) SI_FAIL(SI_ERR_INVALID, "si_gguf_open: cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    SI_FAIL(SI_ERR_INVALID, "si_gguf_open: cannot stat %s", path);
  }
  void* map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  if (map == MAP_FAILED) {
    close(fd);
    SI_FAIL(SI_ERR_INVALID, "si_gguf_open: cannot map %s", path);
  }
  si_gguf* g = new si_gguf();
  g->fd = fd;
  g->map = (const uint8_t*)map;
  g->size = (size_t)st.st_size;
  const int r = parse(g);
  if (r != SI_OK) {
    munmap((void*)g->map, g->size);
    close(fd);
    delete g;
    return r;
  }
  *out = g;
  return SI_OK;
}

SI_EXPORT int si_gguf_close(si_gguf* g) {
  clear_error();
  if (!g) return SI_OK;
  if (g->map) munmap((void*)g->map, g->size);
  if (g->fd >= 0) close(g->fd);
  delete g;
  return SI_OK;
}

SI_EXPORT int si_gguf_info(const si_gguf* g, int* version, int64_t* n_tensors, int64_t* n_kv, int64_t* data_offset) {
  clear_error();
  if (!g) SI_FAIL(SI_ERR_INVALID, "si_gguf_info: NULL file");
  if (version) *version = (int)g->version;
  if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
  if (n_kv) *n_kv = (int64_t)g->kv.size();
  if (data_offset) *data_offset = (int64_t)g->data_off;
  return SI_OK;
}

SI_EXPORT int si_gguf_meta_int(const si_gguf* g, const char* key, int64_t* out) {
  clear_error();
  if (!g || !key || !out) SI_FAIL(SI_ERR_INVALID, "si_gguf_meta_int: NULL argument");
  if (!kv_int(g, key, out)) SI_FAIL(SI_ERR_INVALID, "gguf: no integer key %s", key);
  return SI_OK;
}

SI_EXPORT int si_gguf_meta_float(const si_gguf* g, const char* key, double* out) {
  clear_error();
  if (!g || !key || !out) SI_FAIL(SI_ERR_INVALID, "si_gguf_meta_float: NULL argument");
  if (!kv_float(g, key, out)) SI_FAIL(SI_ERR_INVALID, "gguf: no numeric key %s", key);
  return SI_OK;
}

SI_EXPORT int si_gguf_meta_string(const si_gguf* g, const char* key, char* buf, int len) {
  clear_error();
  if (!g || !key || !buf || len <= 0) SI_FAIL(SI_ERR_INVALID, "si_gguf_meta_string: bad arguments");
  std::string s;
  if (!kv_str(g, key, &s)) SI_FAIL(SI_ERR_INVALID, "gguf: no string key %s", key);
  snprintf(buf, (size_t)len, "%s", s.c_str());
  return SI_OK;
}

SI_EXPORT int si_gguf_meta_array(const si_gguf* g, const char* key, int* item_type, int64_t* count) {
  clear_error();
  if (!g || !key) SI_FAIL(SI_ERR_INVALID, "si_gguf_meta_array: NULL argument");
  const KV* v = find_kv(g, key);
  if (!v || v->type != GT_ARR) SI_FAIL(SI_ERR_INVALID, "gguf: no array key %s", key);
  if (item_type) *item_type = (int)v->item_type;
  if (count) *count = (int64_t)v->count;
  return SI_OK;
}

SI_EXPORT int si_gguf_tensor_info(const si_gguf* g, int64_t i, char* name, int name_len, int* qtype, int64_t* rows,
                                  int64_t* cols, int64_t* bytes) {
  clear_error();
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) SI_FAIL(SI_ERR_INVALID, "si_gguf_tensor_info: index %lld",
                                                              (long long)i);
  const TensorInfo& t = g->tensors[(size_t)i];
  if (name && name_len > 0) snprintf(name, (size_t)name_len, "%s", t.name.c_str());
  uint64_t r = 1;
  for (size_t d = 1; d < t.dims.size(); d++) r *= t.dims[d];
  if (qtype) *qtype = (int)t.type;
  if (rows) *rows = (int64_t)r;
  if (cols) *cols = (int64_t)t.dims[0];
  if (bytes) *bytes = (int64_t)t.bytes;
  return SI_OK;
}

SI_EXPORT int si_gguf_find_tensor(const si_gguf* g, const char* name, int64_t* index) {
  clear_error();
  if (!g || !name || !index) SI_FAIL(SI_ERR_INVALID, "si_gguf_find_tensor: NULL argument");
  auto it = g->by_name.find(name);
  if (it == g->by_name.end()) SI_FAIL(SI_ERR_INVALID, "gguf: no tensor %s", name);
  *index = (int64_t)it->second;
  return SI_OK;
}

SI_EXPORT int si_gguf_tensor_data(const si_gguf* g, int64_t i, const void** data) {
  clear_error();
  if (!g || !data || i < 0 || i >= (int64_t)g->tensors.size())
    SI_FAIL(SI_ERR_INVALID, "si_gguf_tensor_data: bad arguments");
  const TensorInfo& t = g->tensors[(size_t)i];
  if (!t.bytes) SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: tensor %s has ggml type %u", t.name.c_str(), t.type);
  *data = g->map + g->data_off + t.offset;
  return SI_OK;
}

SI_EXPORT int si_gguf_model_config(const si_gguf* g, int max_seq, int max_batch, si_model_config* cfg) {
  clear_error();
  if (!g || !cfg) SI_FAIL(SI_ERR_INVALID, "si_gguf_model_config: NULL argument");
  std::string arch;
  if (!kv_str(g, "general.architecture", &arch)) SI_FAIL(SI_ERR_INVALID, "gguf: no general.architecture");
  if (arch != "llama" && arch != "mistral")
    SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: architecture %s (llama and mistral are read)", arch.c_str());
  int64_t L, h, ff, nh, nkv = -1, hd = -1, ctx = 0;
  if (!kv_int(g, arch + ".block_count", &L) || !kv_int(g, arch + ".embedding_length", &h) ||
      !kv_int(g, arch + ".feed_forward_length", &ff) || !kv_int(g, arch + ".attention.head_count", &nh))
    SI_FAIL(SI_ERR_INVALID, "gguf: %s.block_count / embedding_length / feed_forward_length / head_count missing",
            arch.c_str());
  if (!kv_int(g, arch + ".attention.head_count_kv", &nkv)) nkv = nh;
  if (!kv_int(g, arch + ".attention.key_length", &hd)) hd = nh > 0 ? h / nh : 0;
  kv_int(g, arch + ".context_length", &ctx);
  double eps = 1e-5, theta = 10000.0;
  kv_float(g, arch + ".attention.layer_norm_rms_epsilon", &eps);
  kv_float(g, arch + ".rope.freq_base", &theta);
  const TensorInfo* emb = find_tensor(g, "token_embd.weight");
  if (!emb || emb->dims.size() != 2) SI_FAIL(SI_ERR_INVALID, "gguf: token_embd.weight missing");
  const TensorInfo* out = find_tensor(g, "output.weight");  // absent: tied to the embedding
  const TensorInfo* q0 = find_tensor(g, layer_name(0, SI_T_Q));
  if (!q0) SI_FAIL(SI_ERR_INVALID, "gguf: %s missing", layer_name(0, SI_T_Q).c_str());
  memset(cfg, 0, sizeof(*cfg));
  cfg->n_layers = (int)L;
  cfg->hidden = (int)h;
  cfg->intermediate = (int)ff;
  cfg->n_heads = (int)nh;
  cfg->n_kv_heads = (int)nkv;
  cfg->head_dim = (int)hd;
  cfg->vocab = (int)emb->dims[1];
  cfg->max_seq = max_seq > 0 ? max_seq : (int)ctx;
  cfg->max_batch = max_batch;
  cfg->rms_eps = (float)eps;
  cfg->rope_theta = (float)theta;
  cfg->weight_qtype = (int)q0->type;
  cfg->emb_qtype = (int)emb->type;
  cfg->lm_head_qtype = (int)(out ? out->type : emb->type);
  // every projection must share one supported type (the fused q/k/v and
  // gate/up weights hold one format); norms are f32
  if (!supported_weight(q0->type)) SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: projections of ggml type %u", q0->type);
  for (int l = 0; l < L; l++)
    for (int t = 0; t < 9; t++) {
      const TensorInfo* ti = find_tensor(g, layer_name(l, t));
      if (!ti) SI_FAIL(SI_ERR_INVALID, "gguf: %s missing", layer_name(l, t).c_str());
      const uint32_t want = t >= SI_T_ATTN_NORM ? 0u : q0->type;
      if (ti->type != want)
        SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: %s is ggml type %u, expected %u (projections of one format)",
                ti->name.c_str(), ti->type, want);
    }
  if (!supported_weight(emb->type)) SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: token_embd of ggml type %u", emb->type);
  if (!supported_weight((uint32_t)cfg->lm_head_qtype))
    SI_FAIL(SI_ERR_UNSUPPORTED, "gguf: output of ggml type %d", cfg->lm_head_qtype);
  return SI_OK;
}

SI_EXPORT int si_model_load_gguf(si_model* m, const si_gguf* g) {
  clear_error();
  if (!m || !g) SI_FAIL(SI_ERR_INVALID, "si_model_load_gguf: NULL argument");
  si_model_config fc;
  SI_TRY(si_gguf_model_config(g, 0, 1, &fc));
  si_model_config mc;
  SI_TRY(si_model_get_config(m, &mc));
  if (fc.n_layers != mc.n_layers || fc.hidden != mc.hidden || fc.intermediate != mc.intermediate ||
      fc.n_heads != mc.n_heads || fc.n_kv_heads != mc.n_kv_heads || fc.head_dim != mc.head_dim ||
      fc.vocab != mc.vocab || fc.weight_qtype != mc.weight_qtype || fc.emb_qtype != mc.emb_qtype ||
      fc.lm_head_qtype != mc.lm_head_qtype)
    SI_FAIL(SI_ERR_INVALID, "si_model_load_gguf: the file's configuration differs from the model's");
  auto data = [&](const std::string& name, const void** p) -> int {
    int64_t i;
    SI_TRY(si_gguf_find_tensor(g, name.c_str(), &i));
    return si_gguf_tensor_data(g, i, p);
  };
  for (int l = 0; l < fc.n_layers; l++)
    for (int t = 0; t < 9; t++) {
      const void* p;
      SI_TRY(data(layer_name(l, t), &p));
      SI_TRY(si_model_set_tensor(m, l, t, p));
    }
  const void* p;
  SI_TRY(data("token_embd.weight", &p));
  SI_TRY(si_model_set_tensor(m, -1, SI_T_EMB, p));
  if (find_tensor(g, "output.weight")) SI_TRY(data("output.weight", &p));
  SI_TRY(si_model_set_tensor(m, -1, SI_T_LM_HEAD, p));  // tied embeddings: the same rows
  SI_TRY(data("output_norm.weight", &p));
  SI_TRY(si_model_set_tensor(m, -1, SI_T_FINAL_NORM, p));
  return SI_OK;
}

}  // extern "C"
