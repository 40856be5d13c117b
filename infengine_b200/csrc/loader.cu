// Safetensors weight loader (the reference's
// ModelWeights::from_safetensors, kernels/model_weights.cu:80-154).
//
// The reference parses the header with nlohmann/json, makes one cudaMalloc
// and one blocking copy per tensor and converts bf16 to fp16 in place. Here:
//  * the header is read by a small JSON reader written for the safetensors
//    header (an object of {dtype, shape, data_offsets} objects and an
//    optional "__metadata__" object of strings);
//  * the file is mapped (mmap) and every tensor of one rank goes into ONE
//    device slab (256-byte aligned sub-allocations; per layer the Q, K and V
//    rows are adjacent, a [q+2kv, H] block);
//  * tensor-parallel sharding happens at load: rank r of t keeps its rows of
//    q/k/v/gate/up and of lm_head (vocabulary) and its input columns of o/down
//    (strided 2-D copies); embedding and norms are copied whole;
//  * host data is staged through two pinned buffers so that the file read of
//    one chunk overlaps the host-to-device copy of the previous one; a storage
//    type different from the file's is converted on the device;
//  * the RoPE tables (Llama-3.1 frequency scaling, rope.cu:68-103) are
//    computed on the host in fp32 and uploaded.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <type_traits>
#include <vector>
#include "ie_common.cuh"

namespace {

// ------------------------------------------------------------ JSON reader
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* e;
  int depth = 0;
  bool fail = false;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(e - p) < n || memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  bool string(std::string& out) {
    if (p >= e || *p != '"') return false;
    ++p;
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return false;
        const char x = *p++;
        switch (x) {
          case '"': c = '"'; break;
          case '\\': c = '\\'; break;
          case '/': c = '/'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'n': c = '\n'; break;
          case 'r': c = '\r'; break;
          case 't': c = '\t'; break;
          case 'u': {  // kept as '?': tensor names are ASCII
            if (e - p < 4) return false;
            p += 4;
            c = '?';
            break;
          }
          default: return false;
        }
      }
      out.push_back(c);
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool value(JVal& v) {
    if (++depth > 16) return false;
    ws();
    if (p >= e) return false;
    bool ok = true;
    if (*p == '{') {
      v.kind = JVal::Obj;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
      } else {
        while (ok) {
          ws();
          std::string k;
          JVal x;
          ok = string(k);
          ws();
          ok = ok && p < e && *p++ == ':';
          ok = ok && value(x);
          if (!ok) break;
          v.obj.emplace_back(std::move(k), std::move(x));
          ws();
          if (p < e && *p == ',') { ++p; continue; }
          ok = p < e && *p++ == '}';
          break;
        }
      }
    } else if (*p == '[') {
      v.kind = JVal::Arr;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
      } else {
        while (ok) {
          JVal x;
          ok = value(x);
          if (!ok) break;
          v.arr.push_back(std::move(x));
          ws();
          if (p < e && *p == ',') { ++p; continue; }
          ok = p < e && *p++ == ']';
          break;
        }
      }
    } else if (*p == '"') {
      v.kind = JVal::Str;
      ok = string(v.str);
    } else if (lit("true")) {
      v.kind = JVal::Bool; v.num = 1;
    } else if (lit("false")) {
      v.kind = JVal::Bool;
    } else if (lit("null")) {
      v.kind = JVal::Null;
    } else {
      char* end = nullptr;
      std::string tmp(p, (size_t)(e - p) < 64 ? (size_t)(e - p) : 64);
      v.num = strtod(tmp.c_str(), &end);
      ok = end != tmp.c_str();
      v.kind = JVal::Num;
      p += end - tmp.c_str();
    }
    --depth;
    return ok;
  }
};

// ------------------------------------------------------------ one file
struct Tensor {
  int dtype = 0;  // IE_ST_* code
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte range inside the data section
};

}  // namespace

struct ie_safetensors {
  int fd = -1;
  size_t size = 0;
  const unsigned char* map = nullptr;
  const unsigned char* data = nullptr;  // start of the data section
  std::map<std::string, Tensor> tensors;
  std::vector<std::string> names;
};

namespace {

int dtype_code(const std::string& s) {
  if (s == "BF16") return IE_ST_BF16;
  if (s == "F16") return IE_ST_F16;
  if (s == "F32") return IE_ST_F32;
  return IE_ST_OTHER;
}
size_t dtype_bytes(int code) { return code == IE_ST_F32 ? 4 : 2; }

bool integral(const JVal& v) { return v.kind == JVal::Num && v.num >= 0 && v.num == std::floor(v.num) && v.num < 9.0e15; }

int parse_header(ie_safetensors& f, const char* hdr, size_t n, size_t data_bytes) {
  JParser jp{hdr, hdr + n};
  JVal root;
  if (!jp.value(root) || root.kind != JVal::Obj) return IE_ERR_INVALID_ARG;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal& t = kv.second;
    const JVal* dt = t.get("dtype");
    const JVal* sh = t.get("shape");
    const JVal* off = t.get("data_offsets");
    if (t.kind != JVal::Obj || !dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !off ||
        off->kind != JVal::Arr || off->arr.size() != 2 || !integral(off->arr[0]) || !integral(off->arr[1]))
      return IE_ERR_INVALID_ARG;
    Tensor x;
    x.dtype = dtype_code(dt->str);
    uint64_t elems = 1;
    for (const JVal& d : sh->arr) {
      if (!integral(d)) return IE_ERR_INVALID_ARG;
      const uint64_t dim = (uint64_t)d.num;
      // a shape whose element count wraps around 64 bits could otherwise
      // match a small (or empty) data range
      if (dim != 0 && elems > UINT64_MAX / dim) return IE_ERR_INVALID_ARG;
      x.shape.push_back((int64_t)d.num);
      elems *= dim;
    }
    x.begin = (uint64_t)off->arr[0].num;
    x.end = (uint64_t)off->arr[1].num;
    if (x.end < x.begin || x.end > data_bytes) return IE_ERR_INVALID_ARG;
    if (x.dtype != IE_ST_OTHER && x.end - x.begin != elems * dtype_bytes(x.dtype)) return IE_ERR_INVALID_ARG;
    if (f.tensors.count(kv.first)) return IE_ERR_INVALID_ARG;
    f.tensors[kv.first] = std::move(x);
    f.names.push_back(kv.first);
  }
  return IE_OK;
}

}  // namespace

extern "C" {

int ie_st_open(const char* path, ie_safetensors** out) {
  if (!path || !out) return IE_ERR_INVALID_ARG;
  *out = nullptr;
  ie_safetensors* f = new (std::nothrow) ie_safetensors();
  if (!f) return IE_ERR_INVALID_ARG;
  f->fd = open(path, O_RDONLY);
  struct stat st;
  if (f->fd < 0 || fstat(f->fd, &st) != 0 || st.st_size < 8) {
    ie_st_close(f);
    return IE_ERR_INVALID_ARG;
  }
  f->size = (size_t)st.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) {
    ie_st_close(f);
    return IE_ERR_INVALID_ARG;
  }
  f->map = static_cast<const unsigned char*>(m);
  uint64_t hlen = 0;
  memcpy(&hlen, f->map, 8);  // little-endian u64
  if (hlen > f->size - 8 || hlen > (100u << 20)) {
    ie_st_close(f);
    return IE_ERR_INVALID_ARG;
  }
  f->data = f->map + 8 + hlen;
  const int s = parse_header(*f, reinterpret_cast<const char*>(f->map + 8), hlen, f->size - 8 - hlen);
  if (s != IE_OK) {
    ie_st_close(f);
    return s;
  }
  *out = f;
  return IE_OK;
}

int ie_st_close(ie_safetensors* f) {
  if (!f) return IE_OK;
  if (f->map) munmap(const_cast<unsigned char*>(f->map), f->size);
  if (f->fd >= 0) close(f->fd);
  delete f;
  return IE_OK;
}

int ie_st_count(const ie_safetensors* f) { return f ? (int)f->names.size() : IE_ERR_INVALID_ARG; }

const char* ie_st_name(const ie_safetensors* f, int i) {
  if (!f || i < 0 || i >= (int)f->names.size()) return nullptr;
  return f->names[i].c_str();
}

int ie_st_info(const ie_safetensors* f, const char* name, int* dtype, int* ndim, int64_t* shape,
               uint64_t* nbytes) {
  if (!f || !name) return IE_ERR_INVALID_ARG;
  auto it = f->tensors.find(name);
  if (it == f->tensors.end()) return IE_ERR_INVALID_ARG;
  const Tensor& t = it->second;
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = (int)t.shape.size();
  if (shape)
    for (size_t i = 0; i < t.shape.size() && i < 8; ++i) shape[i] = t.shape[i];
  if (nbytes) *nbytes = t.end - t.begin;
  return IE_OK;
}

}  // extern "C"

// ------------------------------------------------------------ the model
namespace {

template <typename S, typename D>
__global__ void convert_kernel(const S* in, D* out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v;
    if constexpr (std::is_same<S, float>::value) v = in[i];
    else v = ie::DT<S>::to_f(in[i]);
    if constexpr (std::is_same<D, float>::value) out[i] = v;
    else out[i] = ie::DT<D>::from_f(v);
  }
}

struct Source {
  const ie_safetensors* file;
  const Tensor* t;
};

struct Loader {
  ie_dtype dt;
  cudaStream_t st;
  unsigned char* pinned[2] = {nullptr, nullptr};
  size_t chunk = 64u << 20;
  cudaEvent_t done[2] = {nullptr, nullptr};
  int which = 0;
  void* convbuf = nullptr;
  size_t convbytes = 0;
  bool ok = true;

  // rows [r0, r0+nr) x cols [c0, c0+nc) of a row-major [R, C] source tensor
  // into dst (row-major [nr, nc], dt), through the pinned staging buffers.
  int copy(const Source& s, int64_t r0, int64_t nr, int64_t c0, int64_t nc, void* dst) {
    const Tensor& t = *s.t;
    const int64_t C = t.shape.size() == 2 ? t.shape[1] : t.shape[0];
    const size_t sb = dtype_bytes(t.dtype), db = 2;
    const bool same = (t.dtype == IE_ST_BF16 && dt == IE_DTYPE_BF16) || (t.dtype == IE_ST_F16 && dt == IE_DTYPE_F16);
    const size_t row_src = (size_t)nc * sb;
    const int64_t rows_per_chunk = (int64_t)(chunk / row_src) > 0 ? (int64_t)(chunk / row_src) : 1;
    if (row_src > chunk) return IE_ERR_UNSUPPORTED;
    for (int64_t r = 0; r < nr; r += rows_per_chunk) {
      const int64_t n = (nr - r) < rows_per_chunk ? (nr - r) : rows_per_chunk;
      unsigned char* stage = pinned[which];
      if (cudaEventSynchronize(done[which]) != cudaSuccess) return IE_ERR_LAUNCH;
      const unsigned char* src = s.file->data + t.begin + ((size_t)(r0 + r) * C + c0) * sb;
      for (int64_t i = 0; i < n; ++i) memcpy(stage + i * row_src, src + (size_t)i * C * sb, row_src);
      void* target = static_cast<char*>(dst) + (size_t)r * nc * db;
      if (same) {
        if (cudaMemcpyAsync(target, stage, n * row_src, cudaMemcpyHostToDevice, st) != cudaSuccess)
          return IE_ERR_LAUNCH;
      } else {
        if (n * row_src > convbytes) return IE_ERR_UNSUPPORTED;
        if (cudaMemcpyAsync(convbuf, stage, n * row_src, cudaMemcpyHostToDevice, st) != cudaSuccess)
          return IE_ERR_LAUNCH;
        const size_t cnt = (size_t)n * nc;
        const int blocks = (int)((cnt + 255) / 256 < 4096 ? (cnt + 255) / 256 : 4096);
        if (t.dtype == IE_ST_BF16 && dt == IE_DTYPE_F16)
          convert_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(convbuf), static_cast<__half*>(target), cnt);
        else if (t.dtype == IE_ST_F16 && dt == IE_DTYPE_BF16)
          convert_kernel<<<blocks, 256, 0, st>>>(static_cast<const __half*>(convbuf), static_cast<__nv_bfloat16*>(target), cnt);
        else if (t.dtype == IE_ST_F32 && dt == IE_DTYPE_F16)
          convert_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(convbuf), static_cast<__half*>(target), cnt);
        else if (t.dtype == IE_ST_F32 && dt == IE_DTYPE_BF16)
          convert_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(convbuf), static_cast<__nv_bfloat16*>(target), cnt);
        else
          return IE_ERR_UNSUPPORTED;
        // the conversion buffer is reused by the next chunk: keep the order
        if (cudaStreamSynchronize(st) != cudaSuccess) return IE_ERR_LAUNCH;
      }
      if (cudaEventRecord(done[which], st) != cudaSuccess) return IE_ERR_LAUNCH;
      which ^= 1;
    }
    return IE_OK;
  }
};

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Llama-3.1 RoPE tables as init_rope_buffer builds them (rope.cu:68-103):
// theta 500000, factor 8, low/high frequency factors 1 and 4, original
// context 8192; angle = position * frequency in fp32.
void rope_tables(int max_pos, std::vector<float>& cs, std::vector<float>& sn) {
  const int half = 64;
  float freqs[64];
  const double theta = 500000.0, factor = 8.0, lowf = 1.0, highf = 4.0, orig = 8192.0;
  const double low_wl = orig / lowf, high_wl = orig / highf;
  for (int i = 0; i < half; ++i) {
    const float f = (float)(1.0 / std::pow(theta, 2.0 * i / 128.0));
    const float wl = (float)(2.0 * M_PI / (double)f);
    if (wl > low_wl) {
      freqs[i] = f / (float)factor;
    } else if (wl < high_wl) {
      freqs[i] = f;
    } else {
      const float sm = ((float)orig / wl - (float)lowf) / (float)(highf - lowf);
      freqs[i] = (1.0f - sm) * (f / (float)factor) + sm * f;
    }
  }
  cs.resize((size_t)max_pos * half);
  sn.resize((size_t)max_pos * half);
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const float a = (float)p * freqs[i];
      cs[(size_t)p * half + i] = std::cos(a);
      sn[(size_t)p * half + i] = std::sin(a);
    }
}

}  // namespace

struct ie_llama_model {
  ie_llama_desc desc{};
  std::vector<ie_llama_layer_weights> layers;
  void* slab = nullptr;
  int world = 1, rank = 0, lm_rows = 0;
  int64_t lm_offset = 0;
};

extern "C" {

int ie_llama_load(const char* const* paths, int n_paths, ie_dtype dt, int world, int rank, int max_ctx,
                  float rms_eps, void* stream, ie_llama_model** out) {
  if (!out || !paths || n_paths <= 0 || (dt != IE_DTYPE_F16 && dt != IE_DTYPE_BF16) || world < 1 || rank < 0 ||
      rank >= world || max_ctx <= 0)
    return IE_ERR_INVALID_ARG;
  *out = nullptr;
  std::vector<ie_safetensors*> files;
  std::map<std::string, Source> all;
  int s = IE_OK;
  for (int i = 0; i < n_paths && s == IE_OK; ++i) {
    ie_safetensors* f = nullptr;
    s = ie_st_open(paths[i], &f);
    if (s != IE_OK) break;
    files.push_back(f);
    for (const auto& kv : f->tensors) all[kv.first] = Source{f, &kv.second};
  }
  auto cleanup = [&](int status) {
    for (auto* f : files) ie_st_close(f);
    return status;
  };
  if (s != IE_OK) return cleanup(s);
  auto find = [&](const std::string& n) -> const Source* {
    auto it = all.find(n);
    return it == all.end() ? nullptr : &it->second;
  };
  auto layer_name = [](int l, const char* sub) { return "model.layers." + std::to_string(l) + "." + sub; };
  // ---- shapes
  const Source* emb = find("model.embed_tokens.weight");
  const Source* fnorm = find("model.norm.weight");
  const Source* lm = find("lm_head.weight");
  if (!lm) lm = emb;  // tied embeddings
  if (!emb || !fnorm || emb->t->shape.size() != 2) return cleanup(IE_ERR_INVALID_ARG);
  const int64_t V = emb->t->shape[0], H = emb->t->shape[1];
  int L = 0;
  while (find(layer_name(L, "self_attn.q_proj.weight"))) ++L;
  if (L == 0) return cleanup(IE_ERR_INVALID_ARG);
  const Source* q0 = find(layer_name(0, "self_attn.q_proj.weight"));
  const Source* k0 = find(layer_name(0, "self_attn.k_proj.weight"));
  const Source* g0 = find(layer_name(0, "mlp.gate_proj.weight"));
  if (!q0 || !k0 || !g0) return cleanup(IE_ERR_INVALID_ARG);
  const int64_t QD = q0->t->shape[0], KD = k0->t->shape[0], F = g0->t->shape[0];
  if (QD % 128 || KD % 128 || (QD / 128) % world || (KD / 128) % world || F % world || (F / world) % 8 || H % 8)
    return cleanup(IE_ERR_UNSUPPORTED);
  const int64_t qd = QD / world, kd = KD / world, f = F / world;
  const int64_t v0 = V * rank / world, v1 = V * (rank + 1) / world;
  // every tensor must be present with the expected shape
  struct Want { std::string name; int64_t r, c; };
  std::vector<Want> wants = {{"model.embed_tokens.weight", V, H}, {"model.norm.weight", H, 0}};
  for (int l = 0; l < L; ++l) {
    wants.push_back({layer_name(l, "input_layernorm.weight"), H, 0});
    wants.push_back({layer_name(l, "post_attention_layernorm.weight"), H, 0});
    wants.push_back({layer_name(l, "self_attn.q_proj.weight"), QD, H});
    wants.push_back({layer_name(l, "self_attn.k_proj.weight"), KD, H});
    wants.push_back({layer_name(l, "self_attn.v_proj.weight"), KD, H});
    wants.push_back({layer_name(l, "self_attn.o_proj.weight"), H, QD});
    wants.push_back({layer_name(l, "mlp.gate_proj.weight"), F, H});
    wants.push_back({layer_name(l, "mlp.up_proj.weight"), F, H});
    wants.push_back({layer_name(l, "mlp.down_proj.weight"), H, F});
  }
  for (const Want& w : wants) {
    const Source* x = find(w.name);
    if (!x || x->t->dtype == IE_ST_OTHER) return cleanup(IE_ERR_INVALID_ARG);
    const auto& sh = x->t->shape;
    const bool ok = w.c ? (sh.size() == 2 && sh[0] == w.r && sh[1] == w.c) : (sh.size() == 1 && sh[0] == w.r);
    if (!ok) return cleanup(IE_ERR_INVALID_ARG);
  }
  if (lm->t->shape.size() != 2 || lm->t->shape[0] != V || lm->t->shape[1] != H) return cleanup(IE_ERR_INVALID_ARG);
  // ---- slab layout (elements of dt, 256-byte aligned pieces)
  size_t off = 0;
  auto take = [&](size_t elems) {
    const size_t o = off;
    off = align256(off + elems * 2);
    return o;
  };
  const size_t o_emb = take((size_t)V * H), o_fnorm = take(H), o_lm = take((size_t)(v1 - v0) * H);
  struct LOff { size_t an, fn, qkv, o, g, u, d; };
  std::vector<LOff> lo(L);
  for (int l = 0; l < L; ++l) {
    lo[l].an = take(H);
    lo[l].fn = take(H);
    lo[l].qkv = take((size_t)(qd + 2 * kd) * H);  // Q, K, V rows adjacent
    lo[l].o = take((size_t)H * qd);
    lo[l].g = take((size_t)f * H);
    lo[l].u = take((size_t)f * H);
    lo[l].d = take((size_t)H * f);
  }
  const size_t o_cos = take((size_t)max_ctx * 64 * 2);  // fp32 tables: 2 x 2-byte units per value
  const size_t o_sin = take((size_t)max_ctx * 64 * 2);
  ie_llama_model* m = new (std::nothrow) ie_llama_model();
  if (!m) return cleanup(IE_ERR_INVALID_ARG);
  Loader ld;
  ld.dt = dt;
  ld.st = static_cast<cudaStream_t>(stream);
  ld.convbytes = ld.chunk;
  bool ok = cudaMalloc(&m->slab, off) == cudaSuccess && cudaMallocHost((void**)&ld.pinned[0], ld.chunk) == cudaSuccess &&
            cudaMallocHost((void**)&ld.pinned[1], ld.chunk) == cudaSuccess &&
            cudaMalloc(&ld.convbuf, ld.convbytes) == cudaSuccess && cudaEventCreate(&ld.done[0]) == cudaSuccess &&
            cudaEventCreate(&ld.done[1]) == cudaSuccess;
  auto at = [&](size_t o) { return static_cast<void*>(static_cast<char*>(m->slab) + o); };
  s = ok ? IE_OK : IE_ERR_WORKSPACE;
  if (ok) cudaEventRecord(ld.done[0], ld.st), cudaEventRecord(ld.done[1], ld.st);
  auto full = [&](const std::string& n, size_t o) {
    const Source* x = find(n);
    const auto& sh = x->t->shape;
    return sh.size() == 2 ? ld.copy(*x, 0, sh[0], 0, sh[1], at(o)) : ld.copy(*x, 0, 1, 0, sh[0], at(o));
  };
  if (s == IE_OK) s = full("model.embed_tokens.weight", o_emb);
  if (s == IE_OK) s = full("model.norm.weight", o_fnorm);
  if (s == IE_OK) s = ld.copy(*lm, v0, v1 - v0, 0, H, at(o_lm));
  for (int l = 0; l < L && s == IE_OK; ++l) {
    const LOff& x = lo[l];
    s = full(layer_name(l, "input_layernorm.weight"), x.an);
    if (s == IE_OK) s = full(layer_name(l, "post_attention_layernorm.weight"), x.fn);
    if (s == IE_OK) s = ld.copy(*find(layer_name(l, "self_attn.q_proj.weight")), rank * qd, qd, 0, H, at(x.qkv));
    if (s == IE_OK)
      s = ld.copy(*find(layer_name(l, "self_attn.k_proj.weight")), rank * kd, kd, 0, H, at(x.qkv + qd * H * 2));
    if (s == IE_OK)
      s = ld.copy(*find(layer_name(l, "self_attn.v_proj.weight")), rank * kd, kd, 0, H,
                  at(x.qkv + (qd + kd) * H * 2));
    if (s == IE_OK) s = ld.copy(*find(layer_name(l, "self_attn.o_proj.weight")), 0, H, rank * qd, qd, at(x.o));
    if (s == IE_OK) s = ld.copy(*find(layer_name(l, "mlp.gate_proj.weight")), rank * f, f, 0, H, at(x.g));
    if (s == IE_OK) s = ld.copy(*find(layer_name(l, "mlp.up_proj.weight")), rank * f, f, 0, H, at(x.u));
    if (s == IE_OK) s = ld.copy(*find(layer_name(l, "mlp.down_proj.weight")), 0, H, rank * f, f, at(x.d));
  }
  if (s == IE_OK) {
    std::vector<float> cs, sn;
    rope_tables(max_ctx, cs, sn);
    if (cudaMemcpyAsync(at(o_cos), cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, ld.st) != cudaSuccess ||
        cudaMemcpyAsync(at(o_sin), sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, ld.st) != cudaSuccess ||
        cudaStreamSynchronize(ld.st) != cudaSuccess)
      s = IE_ERR_LAUNCH;
  }
  if (ld.pinned[0]) cudaFreeHost(ld.pinned[0]);
  if (ld.pinned[1]) cudaFreeHost(ld.pinned[1]);
  if (ld.convbuf) cudaFree(ld.convbuf);
  if (ld.done[0]) cudaEventDestroy(ld.done[0]);
  if (ld.done[1]) cudaEventDestroy(ld.done[1]);
  if (s != IE_OK) {
    if (m->slab) cudaFree(m->slab);
    delete m;
    cudaGetLastError();
    return cleanup(s);
  }
  m->world = world;
  m->rank = rank;
  m->lm_rows = (int)(v1 - v0);
  m->lm_offset = v0;
  m->layers.resize(L);
  for (int l = 0; l < L; ++l) {
    const LOff& x = lo[l];
    m->layers[l] = ie_llama_layer_weights{at(x.an), at(x.qkv), at(x.qkv + qd * H * 2), at(x.qkv + (qd + kd) * H * 2),
                                          at(x.o), at(x.fn), at(x.g), at(x.u), at(x.d)};
  }
  ie_llama_desc& d = m->desc;
  d.n_layers = L;
  d.hidden = (int)H;
  d.n_q_heads = (int)(qd / 128);
  d.n_kv_heads = (int)(kd / 128);
  d.head_dim = 128;
  d.ffn_dim = (int)f;
  d.vocab = (int)V;
  d.rms_eps = rms_eps;
  d.embedding = at(o_emb);
  d.layers = m->layers.data();
  d.final_norm = at(o_fnorm);
  d.lm_head = at(o_lm);
  d.rope_cos = static_cast<const float*>(at(o_cos));
  d.rope_sin = static_cast<const float*>(at(o_sin));
  *out = m;
  return cleanup(IE_OK);
}

const ie_llama_desc* ie_llama_model_desc(const ie_llama_model* m) { return m ? &m->desc : nullptr; }

int ie_llama_model_shard(const ie_llama_model* m, int* lm_rows, int64_t* lm_offset) {
  if (!m) return IE_ERR_INVALID_ARG;
  if (lm_rows) *lm_rows = m->lm_rows;
  if (lm_offset) *lm_offset = m->lm_offset;
  return IE_OK;
}

int ie_llama_model_free(ie_llama_model* m) {
  if (!m) return IE_OK;
  if (m->slab) cudaFree(m->slab);
  delete m;
  return IE_OK;
}

}  // extern "C"
