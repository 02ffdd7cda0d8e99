// Checkpoints: a safetensors reader (memory-mapped shards, merged in the caller's order) and
// the Whisper loader that fills a vella_whisper handle from a Hugging Face or mlx-whisper
// checkpoint, quantizing float Linears at load when the handle is int4/int8.
//
// Replaces MLX.loadArrays over a model directory's *.safetensors files, merged in file-name
// order with later keys winning (Worker/Sources/MLXAudioSTT/Whisper/WhisperModel.swift:
// 676-684), and the Whisper key sanitising of WhisperModel.sanitize / sanitizeHuggingFace /
// sanitizeMlxWhisper / remapMlxWhisperKey (:483-651): format detection by ".blocks.", the
// tied proj_out dropped, a missing "model." prefix added, PyTorch Conv1d [out, in, k] taken
// as [out, k, in], the OpenAI/mlx-whisper names mapped onto the Hugging Face ones; then the
// derived precision (:686-701: every decoder Linear and the token embedding MLX-affine
// quantized from the float source, positional tables float) or an already-quantized
// checkpoint's packed weights, scales and biases (group 64).
//
// Only the public C ABI of the handle is used: vella_whisper_get_cfg, vella_whisper_tensor
// (device pointers of every tensor) and vella_quantize.  All of this is load-time host code.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <initializer_list>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <type_traits>
#include <unordered_map>
#include <utility>
#include <vector>

#include "internal.h"
#include "vella_cuda.h"

using vella::fail;

namespace {

// ---- a small JSON reader for safetensors headers ---------------------------------------

struct JVal {
  enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  long long i = 0;
  double d = 0.0;
  std::string s;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* key) const {
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* p, const char* e) : p_(p), e_(e) {}
  bool parse(JVal& v) {
    if (!value(v, 0)) return false;
    ws();
    return p_ == e_;
  }

 private:
  const char *p_, *e_;
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(e_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) {
      o += (char)c;
    } else if (c < 0x800) {
      o += (char)(0xC0 | (c >> 6));
      o += (char)(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      o += (char)(0xE0 | (c >> 12));
      o += (char)(0x80 | ((c >> 6) & 0x3F));
      o += (char)(0x80 | (c & 0x3F));
    } else {
      o += (char)(0xF0 | (c >> 18));
      o += (char)(0x80 | ((c >> 12) & 0x3F));
      o += (char)(0x80 | ((c >> 6) & 0x3F));
      o += (char)(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t& c) {
    if (e_ - p_ < 4) return false;
    c = 0;
    for (int k = 0; k < 4; ++k) {
      const char h = *p_++;
      c <<= 4;
      if (h >= '0' && h <= '9') c |= (uint32_t)(h - '0');
      else if (h >= 'a' && h <= 'f') c |= (uint32_t)(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') c |= (uint32_t)(h - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool str(std::string& o) {
    if (p_ >= e_ || *p_ != '"') return false;
    ++p_;
    while (p_ < e_ && *p_ != '"') {
      const char c = *p_++;
      if ((unsigned char)c < 0x20) return false;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p_ >= e_) return false;
      const char x = *p_++;
      switch (x) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2;
            if (!lit("\\u") || !hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000) return false;
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          utf8(o, c1);
          break;
        }
        default: return false;
      }
    }
    if (p_ >= e_) return false;
    ++p_;
    return true;
  }
  bool num(JVal& v) {
    const char* s = p_;
    if (p_ < e_ && *p_ == '-') ++p_;
    bool frac = false;
    while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                       *p_ == '-')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') frac = true;
      ++p_;
    }
    if (p_ == s) return false;
    const std::string t(s, p_);
    char* end = nullptr;
    if (!frac) {
      errno = 0;
      v.kind = JVal::Int;
      v.i = std::strtoll(t.c_str(), &end, 10);
      v.d = (double)v.i;
      return errno == 0 && end && *end == '\0';
    }
    v.kind = JVal::Num;
    v.d = std::strtod(t.c_str(), &end);
    return end && *end == '\0';
  }
  bool value(JVal& v, int depth) {
    if (depth > 64) return false;
    ws();
    if (p_ >= e_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.kind = JVal::Obj;
      ws();
      if (p_ < e_ && *p_ == '}') { ++p_; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return false;
        ++p_;
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == '}') { ++p_; return true; }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      v.kind = JVal::Arr;
      ws();
      if (p_ < e_ && *p_ == ']') { ++p_; return true; }
      for (;;) {
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.arr.push_back(std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') { ++p_; continue; }
        if (p_ < e_ && *p_ == ']') { ++p_; return true; }
        return false;
      }
    }
    if (c == '"') {
      v.kind = JVal::Str;
      return str(v.s);
    }
    if (lit("true")) { v.kind = JVal::Bool; v.b = true; return true; }
    if (lit("false")) { v.kind = JVal::Bool; return true; }
    if (lit("null")) { v.kind = JVal::Null; return true; }
    return num(v);
  }
};

// ---- safetensors ------------------------------------------------------------------------

struct StDtype {
  const char* name;
  int code;
  int size;
};
const StDtype kStDtypes[] = {
    {"BF16", VELLA_ST_BF16, 2}, {"F16", VELLA_ST_F16, 2},  {"F32", VELLA_ST_F32, 4},
    {"U32", VELLA_ST_U32, 4},   {"I32", VELLA_ST_I32, 4},  {"U8", VELLA_ST_U8, 1},
    {"I8", VELLA_ST_I8, 1},     {"I64", VELLA_ST_I64, 8},  {"F64", VELLA_ST_F64, 8},
    {"U16", VELLA_ST_U16, 2},   {"I16", VELLA_ST_I16, 2},  {"BOOL", VELLA_ST_BOOL, 1},
    {"U64", VELLA_ST_U64, 8},   {"F8_E4M3", VELLA_ST_F8_E4M3, 1}, {"F8_E5M2", VELLA_ST_F8_E5M2, 1},
};

struct StMap {
  void* base = nullptr;
  size_t size = 0;
  ~StMap() {
    if (base) munmap(base, size);
  }
};

struct StEntry {
  std::string name;
  int dtype = -1, esize = 0;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  int file = 0;
  size_t numel() const {
    size_t n = 1;
    for (int64_t d : shape) n *= (size_t)d;
    return n;
  }
};

}  // namespace

struct vella_st {
  std::vector<std::unique_ptr<StMap>> maps;
  std::vector<StEntry> entries;
  std::unordered_map<std::string, int> index;
  const StEntry* find(const std::string& k) const {
    const auto it = index.find(k);
    return it == index.end() ? nullptr : &entries[(size_t)it->second];
  }
};

namespace {

int st_add_file(vella_st* st, const char* path) {
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(VELLA_E_INVALID, "vella_st_open: cannot open '%s'", path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    close(fd);
    return fail(VELLA_E_INVALID, "vella_st_open: '%s' is not a safetensors file (size)", path);
  }
  auto map = std::make_unique<StMap>();
  map->size = (size_t)sb.st_size;
  void* base = mmap(nullptr, map->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (base == MAP_FAILED) return fail(VELLA_E_INVALID, "vella_st_open: cannot map '%s'", path);
  map->base = base;
  const uint8_t* b = static_cast<const uint8_t*>(base);
  uint64_t hlen = 0;
  for (int k = 7; k >= 0; --k) hlen = (hlen << 8) | b[k];  // little-endian u64
  if (hlen > map->size - 8 || hlen > (100ull << 20))
    return fail(VELLA_E_INVALID, "vella_st_open: '%s': header of %llu bytes in a %zu-byte file", path,
                (unsigned long long)hlen, map->size);
  JVal root;
  const char* h = reinterpret_cast<const char*>(b + 8);
  if (!JParser(h, h + hlen).parse(root) || root.kind != JVal::Obj)
    return fail(VELLA_E_INVALID, "vella_st_open: '%s': the header is not a JSON object", path);
  const uint8_t* data = b + 8 + hlen;
  const size_t dsize = map->size - 8 - (size_t)hlen;
  const int file = (int)st->maps.size();
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal& t = kv.second;
    const JVal* dt = t.get("dtype");
    const JVal* sh = t.get("shape");
    const JVal* off = t.get("data_offsets");
    if (t.kind != JVal::Obj || !dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !off ||
        off->kind != JVal::Arr || off->arr.size() != 2 || off->arr[0].kind != JVal::Int ||
        off->arr[1].kind != JVal::Int)
      return fail(VELLA_E_INVALID, "vella_st_open: '%s': malformed entry '%s'", path, kv.first.c_str());
    StEntry e;
    e.name = kv.first;
    for (const StDtype& d : kStDtypes)
      if (dt->s == d.name) { e.dtype = d.code; e.esize = d.size; }
    if (e.dtype < 0)
      return fail(VELLA_E_INVALID, "vella_st_open: '%s': tensor '%s' has dtype %s", path, kv.first.c_str(),
                  dt->s.c_str());
    if (sh->arr.size() > 8) return fail(VELLA_E_INVALID, "vella_st_open: '%s': rank > 8", kv.first.c_str());
    for (const JVal& d : sh->arr) {
      if (d.kind != JVal::Int || d.i < 0) return fail(VELLA_E_INVALID, "vella_st_open: '%s': bad shape", kv.first.c_str());
      e.shape.push_back(d.i);
    }
    // the element count times the element size must not overflow (a huge shape over a few bytes)
    unsigned long long n = (unsigned long long)e.esize;
    bool overflow = false;
    for (int64_t d : e.shape) {
      if (d != 0 && n > ~0ull / (unsigned long long)d) overflow = true;
      n *= (unsigned long long)d;
    }
    const long long lo = off->arr[0].i, hi = off->arr[1].i;
    if (overflow || lo < 0 || hi < lo || (unsigned long long)hi > dsize || (unsigned long long)(hi - lo) != n)
      return fail(VELLA_E_INVALID, "vella_st_open: '%s': tensor '%s' offsets [%lld, %lld) do not fit its shape or the file",
                  path, kv.first.c_str(), lo, hi);
    e.data = data + lo;
    e.bytes = (size_t)(hi - lo);
    e.file = file;
    const auto it = st->index.find(e.name);
    if (it != st->index.end()) {
      st->entries[(size_t)it->second] = std::move(e);  // a later shard replaces the key
    } else {
      st->index.emplace(e.name, (int)st->entries.size());
      st->entries.push_back(std::move(e));
    }
  }
  st->maps.push_back(std::move(map));
  return VELLA_OK;
}

// ---- Whisper key mapping -----------------------------------------------------------------

bool starts(const std::string& s, const char* p) { return s.rfind(p, 0) == 0; }

// OpenAI / mlx-whisper block suffix -> Hugging Face suffix ("" when the key is not a model
// parameter).  attn.{query,key,value,out} -> self_attn.{q,k,v,out}_proj; cross_attn.* ->
// encoder_attn.*; attn_ln / cross_attn_ln / mlp_ln -> the three LayerNorms; mlp1/mlp2 -> fc1/fc2.
std::string mlx_block_suffix(const std::string& s, bool decoder) {
  static const std::pair<const char*, const char*> proj[] = {
      {"query.", "q_proj."}, {"key.", "k_proj."}, {"value.", "v_proj."}, {"out.", "out_proj."}};
  auto attn = [&](const std::string& rest, const char* container) -> std::string {
    for (const auto& pp : proj)
      if (starts(rest, pp.first)) return std::string(container) + "." + pp.second + rest.substr(std::strlen(pp.first));
    return "";
  };
  if (starts(s, "attn_ln.")) return "self_attn_layer_norm." + s.substr(8);
  if (decoder && starts(s, "cross_attn_ln.")) return "encoder_attn_layer_norm." + s.substr(14);
  if (starts(s, "mlp_ln.")) return "final_layer_norm." + s.substr(7);
  if (starts(s, "mlp1.")) return "fc1." + s.substr(5);
  if (starts(s, "mlp2.")) return "fc2." + s.substr(5);
  if (starts(s, "attn.")) return attn(s.substr(5), "self_attn");
  if (decoder && starts(s, "cross_attn.")) return attn(s.substr(11), "encoder_attn");
  return "";
}

std::string mlx_key(const std::string& k) {
  if (k == "encoder.positional_embedding") return "model.encoder.embed_positions.weight";
  if (k == "decoder.positional_embedding") return "model.decoder.embed_positions.weight";
  if (starts(k, "decoder.token_embedding.")) return "model.decoder.embed_tokens." + k.substr(24);
  if (starts(k, "encoder.conv1.") || starts(k, "encoder.conv2.")) return "model." + k;
  if (starts(k, "encoder.ln_post.")) return "model.encoder.layer_norm." + k.substr(16);
  if (starts(k, "decoder.ln.")) return "model.decoder.layer_norm." + k.substr(11);
  for (const char* stem : {"encoder", "decoder"}) {
    const std::string pre = std::string(stem) + ".blocks.";
    if (!starts(k, pre.c_str())) continue;
    const std::string rest = k.substr(pre.size());
    const size_t dot = rest.find('.');
    if (dot == std::string::npos) return "";
    const std::string suf = mlx_block_suffix(rest.substr(dot + 1), stem[0] == 'd');
    if (suf.empty()) return "";
    return "model." + std::string(stem) + ".layers." + rest.substr(0, dot) + "." + suf;
  }
  return "";
}

std::string hf_key(const std::string& k) {
  if (k == "proj_out.weight" || k == "model.proj_out.weight") return "";  // tied to embed_tokens
  if (!starts(k, "model.") && (starts(k, "encoder.") || starts(k, "decoder."))) return "model." + k;
  return k;
}

// Canonical (Hugging Face) name -> entry, and whether conv weights are PyTorch [out, in, k].
struct KeyView {
  std::unordered_map<std::string, const StEntry*> by;
  std::unordered_map<std::string, bool> transposed;  // stacked experts stored [E][in][out] (NeMo)
  bool hf = true;
  bool quantized = false;  // some tensor has MLX-affine scales (an already-quantized checkpoint)
  const StEntry* get(const std::string& k) const {
    const auto it = by.find(k);
    return it == by.end() ? nullptr : it->second;
  }
};

KeyView whisper_view(const vella_st* st) {
  KeyView v;
  for (const StEntry& e : st->entries)
    if (e.name.find(".blocks.") != std::string::npos) v.hf = false;
  for (const StEntry& e : st->entries) {
    if (!v.hf && e.name == "alignment_heads") continue;
    const std::string k = v.hf ? hf_key(e.name) : mlx_key(e.name);
    if (k.empty()) continue;
    v.by[k] = &e;
    if (k.size() > 7 && k.compare(k.size() - 7, 7, ".scales") == 0) v.quantized = true;
  }
  return v;
}

// ---- element conversion -------------------------------------------------------------------

float elem_f(const StEntry& e, size_t i) {
  const uint8_t* p = e.data + i * (size_t)e.esize;
  switch (e.dtype) {
    case VELLA_ST_F32: { float f; std::memcpy(&f, p, 4); return f; }
    case VELLA_ST_F16: { __half h; std::memcpy(&h, p, 2); return __half2float(h); }
    case VELLA_ST_BF16: { __nv_bfloat16 h; std::memcpy(&h, p, 2); return __bfloat162float(h); }
    default: return 0.0f;
  }
}
bool is_float(const StEntry& e) {
  return e.dtype == VELLA_ST_F32 || e.dtype == VELLA_ST_F16 || e.dtype == VELLA_ST_BF16;
}
uint16_t act_bits(float v, int act) {
  uint16_t o;
  if (act == VELLA_F16) {
    const __half h = __float2half_rn(v);
    std::memcpy(&o, &h, 2);
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    std::memcpy(&o, &h, 2);
  }
  return o;
}

// ---- MLX-affine rows back to the activation dtype ------------------------------------------

template <typename T>
__device__ __forceinline__ float act_to_f(T v) {
  if constexpr (std::is_same<T, __half>::value) return __half2float(v);
  else return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T act_from_f(float v) {
  if constexpr (std::is_same<T, __half>::value) return __float2half_rn(v);
  else return __float2bfloat16_rn(v);
}

// out[r, k] = T(scale * q + bias) for a packed [N, K*bits/32] weight with [N, K/64] scales and
// biases: the multiply and the add each rounded to fp32, then one rounding to T (the value the
// tensor-core GEMM dequantizes a weight to).
template <typename T>
__global__ void __launch_bounds__(256) dequant_rows_kernel(T* __restrict__ out, const uint32_t* __restrict__ packed,
                                                           const T* __restrict__ s, const T* __restrict__ b,
                                                           int64_t K, int bits, int64_t n) {
  const int per = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K, k = i % K;
    const uint32_t q = (packed[r * (K / per) + k / per] >> ((int)(k % per) * bits)) & mask;
    const int64_t g = r * (K / 64) + k / 64;
    out[i] = act_from_f<T>(__fadd_rn(__fmul_rn(act_to_f(s[g]), (float)q), act_to_f(b[g])));
  }
}

// ---- the loader --------------------------------------------------------------------------

// Checks (no `tensor` callback) or fills a handle's tensors from checkpoint entries; the
// callback is the handle's tensor lookup (name, layer) -> device pointer and size.
using TensorFn = std::function<int(const char*, int, void**, size_t*)>;

struct Loader {
  TensorFn tensor;  // empty: check only
  const KeyView& v;
  int act;
  cudaStream_t stream = nullptr;
  bool w = false;   // filling (true) or checking
  // > 0: float Linears of a dense part of the handle hold their MLX-affine values at these
  // bits (quantized, then dequantized), as the reference's derived precision quantizes them
  int fake_bits = 0;

  int dest(const std::string& name, int layer, size_t want, void** p) {
    if (!w) return VELLA_OK;
    size_t bytes = 0;
    int rc = tensor(name.c_str(), layer, p, &bytes);
    if (rc) return rc;
    if (bytes != want)
      return fail(VELLA_E_INVALID, "checkpoint load: '%s' holds %zu bytes, expected %zu", name.c_str(), bytes, want);
    return VELLA_OK;
  }
  int put(void* d, const void* h, size_t bytes) {
    if (!w) return VELLA_OK;
    VELLA_CUDA_TRY(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, stream));
    VELLA_CUDA_TRY(cudaStreamSynchronize(stream));  // the host buffer dies with the caller
    return VELLA_OK;
  }
  const StEntry* need(const std::string& k) {
    const StEntry* e = v.get(k);
    if (!e) fail(VELLA_E_INVALID, "checkpoint: missing '%s'", k.c_str());
    return e;
  }
  static bool shape_is(const StEntry* e, std::initializer_list<int64_t> s) {
    return e->shape.size() == s.size() && std::equal(s.begin(), s.end(), e->shape.begin());
  }

  // a [n] float vector (LayerNorm weight or bias)
  int vec(const std::string& dname, int layer, const std::string& key, int64_t n) {
    const StEntry* e = need(key);
    if (!e) return VELLA_E_INVALID;
    if (!is_float(*e) || !shape_is(e, {n}))
      return fail(VELLA_E_INVALID, "checkpoint: '%s' must be a float [%lld]", key.c_str(), (long long)n);
    void* d = nullptr;
    int rc = dest(dname, layer, (size_t)n * 2, &d);
    if (rc || !w) return rc;
    std::vector<uint16_t> h((size_t)n);
    for (int64_t i = 0; i < n; ++i) h[(size_t)i] = act_bits(elem_f(*e, (size_t)i), act);
    return put(d, h.data(), h.size() * 2);
  }

  // a float tensor of n elements (any of `shapes`) into an fp32 destination (routers, A_log, D, dt_bias)
  int f32(const std::string& dname, int layer, const std::string& key, int64_t n) {
    const StEntry* e = need(key);
    if (!e) return VELLA_E_INVALID;
    if (!is_float(*e) || (int64_t)e->numel() != n)
      return fail(VELLA_E_INVALID, "checkpoint: '%s' must be a float tensor of %lld elements", key.c_str(), (long long)n);
    void* d = nullptr;
    int rc = dest(dname, layer, (size_t)n * 4, &d);
    if (rc || !w) return rc;
    std::vector<float> h((size_t)n);
    for (int64_t i = 0; i < n; ++i) h[(size_t)i] = elem_f(*e, (size_t)i);
    return put(d, h.data(), h.size() * 4);
  }

  // a float tensor of n elements into an activation-dtype destination, element order kept (a
  // [C, 1, K] or [C, K, 1] depthwise conv weight is [C][K] in memory either way)
  int flat(const std::string& dname, int layer, const std::string& key, int64_t n) {
    const StEntry* e = need(key);
    if (!e) return VELLA_E_INVALID;
    if (!is_float(*e) || (int64_t)e->numel() != n)
      return fail(VELLA_E_INVALID, "checkpoint: '%s' must be a float tensor of %lld elements", key.c_str(), (long long)n);
    void* d = nullptr;
    int rc = dest(dname, layer, (size_t)n * 2, &d);
    if (rc || !w) return rc;
    std::vector<uint16_t> h((size_t)n);
    for (int64_t i = 0; i < n; ++i) h[(size_t)i] = act_bits(elem_f(*e, (size_t)i), act);
    return put(d, h.data(), h.size() * 2);
  }

  // stacked experts [E][N][K] (or [E][K][N] when the view marks the key transposed): float
  // (quantized at load for an int handle, or stored dense), or MLX-affine at the handle's bits
  int experts(const std::string& dname, int layer, const std::string& key, int64_t E, int64_t N, int64_t K, int bits) {
    const StEntry* W = need(key + ".weight");
    if (!W) return VELLA_E_INVALID;
    const StEntry* S = v.get(key + ".scales");
    const StEntry* B = v.get(key + ".biases");
    const auto ti = v.transposed.find(key + ".weight");
    const bool tr = ti != v.transposed.end() && ti->second;
    const size_t wb = bits ? (size_t)(E * N) * (size_t)(K * bits / 32) * 4 : (size_t)(E * N * K) * 2;
    const size_t sb = bits ? (size_t)(E * N) * (size_t)(K / 64) * 2 : 0;
    if (S) {
      if (tr || !B || W->dtype != VELLA_ST_U32 || !bits || !shape_is(W, {E, N, K * bits / 32}) ||
          !shape_is(S, {E, N, K / 64}) || !shape_is(B, {E, N, K / 64}) || !is_float(*S) || !is_float(*B))
        return fail(VELLA_E_UNSUPPORTED, "checkpoint: '%s' must be MLX-affine [%lld, %lld, %lld] at %d bits",
                    key.c_str(), (long long)E, (long long)N, (long long)K, bits);
      void *dw = nullptr, *ds = nullptr, *db = nullptr;
      int rc;
      if ((rc = dest(dname + ".w", layer, wb, &dw)) || (rc = dest(dname + ".s", layer, sb, &ds)) ||
          (rc = dest(dname + ".b", layer, sb, &db)) || !w)
        return rc;
      std::vector<uint16_t> hs(sb / 2), hb(sb / 2);
      for (size_t g = 0; g < hs.size(); ++g) {
        hs[g] = act_bits(elem_f(*S, g), act);
        hb[g] = act_bits(elem_f(*B, g), act);
      }
      if ((rc = put(dw, W->data, wb)) || (rc = put(ds, hs.data(), sb))) return rc;
      return put(db, hb.data(), sb);
    }
    if (!is_float(*W) || !(tr ? shape_is(W, {E, K, N}) : shape_is(W, {E, N, K})))
      return fail(VELLA_E_INVALID, "checkpoint: '%s.weight' must be a float [%lld, %lld, %lld]%s", key.c_str(),
                  (long long)E, (long long)(tr ? K : N), (long long)(tr ? N : K), tr ? " (in, out)" : "");
    if (!w) {
      void* dummy = nullptr;
      return dest(dname + ".w", layer, wb, &dummy);
    }
    // [E * N][K] rows in fp32 (transposed when needed), then dense or quantized at load
    std::vector<float> rows((size_t)(E * N * K));
    for (int64_t e = 0; e < E; ++e)
      for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k)
          rows[(size_t)((e * N + n) * K + k)] = elem_f(*W, tr ? (size_t)((e * K + k) * N + n) : (size_t)((e * N + n) * K + k));
    void *dw = nullptr, *ds = nullptr, *db = nullptr;
    int rc;
    if ((rc = dest(dname + ".w", layer, wb, &dw))) return rc;
    if (!bits) {
      std::vector<uint16_t> h(rows.size());
      for (size_t i = 0; i < rows.size(); ++i) h[i] = act_bits(rows[i], act);
      return put(dw, h.data(), h.size() * 2);
    }
    if ((rc = dest(dname + ".s", layer, sb, &ds)) || (rc = dest(dname + ".b", layer, sb, &db))) return rc;
    void* tmp = nullptr;
    VELLA_CUDA_TRY(cudaMalloc(&tmp, rows.size() * 4));
    vella_qgemm_desc qd{};
    qd.m = 1; qd.n = (int32_t)(E * N); qd.k = (int32_t)K; qd.bits = bits; qd.group_size = 64; qd.dtype = act;
    cudaError_t ce = cudaMemcpyAsync(tmp, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, stream);
    if (ce == cudaSuccess) {
      rc = vella_quantize(&qd, VELLA_F32, tmp, dw, ds, db, stream);
      ce = cudaStreamSynchronize(stream);
    }
    cudaFree(tmp);
    if (rc) return rc;
    return ce == cudaSuccess ? VELLA_OK : vella::cuda_fail(ce, "checkpoint load: quantize experts");
  }

  // a [rows, d] position table: the first `rows` rows of the checkpoint's table
  int table(const std::string& dname, const std::string& key, int64_t rows, int64_t dm, bool optional) {
    const StEntry* e = v.get(key);
    if (!e) return optional ? VELLA_OK : fail(VELLA_E_INVALID, "checkpoint: missing '%s'", key.c_str());
    if (!is_float(*e) || e->shape.size() != 2 || e->shape[0] < rows || e->shape[1] != dm)
      return fail(VELLA_E_INVALID, "checkpoint: '%s' must be a float [>= %lld, %lld]", key.c_str(),
                  (long long)rows, (long long)dm);
    void* d = nullptr;
    int rc = dest(dname, -1, (size_t)(rows * dm) * 2, &d);
    if (rc || !w) return rc;
    std::vector<uint16_t> h((size_t)(rows * dm));
    for (size_t i = 0; i < h.size(); ++i) h[i] = act_bits(elem_f(*e, i), act);
    return put(d, h.data(), h.size() * 2);
  }

  // One Linear of the handle from row blocks of checkpoint Linears (q|k|v, k|v), each
  // `prefix.weight` float [n, K] or MLX-affine (`prefix.weight` u32 [n, K*b/32] with
  // `.scales`/`.biases` [n, K/64]).  `bits` is the handle's (0 = dense); `kpad` pads dense
  // columns with zeros; `conv` reads a Conv1d weight (k = 3) into columns j*C + c.
  struct Part {
    std::string prefix;
    int64_t rows;
    bool bias;  // false: the bias rows are zero (k_proj)
  };
  int linear(const std::string& dname, int layer, const std::vector<Part>& parts, int64_t K, int bits,
             int64_t kpad, bool conv, bool with_bias) {
    int64_t N = 0;
    for (const Part& p : parts) N += p.rows;
    int qbits = -1;  // checkpoint packing of the parts: -1 unknown, 0 float, 4 | 8
    std::vector<const StEntry*> W(parts.size()), S(parts.size()), B(parts.size()), Bias(parts.size());
    for (size_t i = 0; i < parts.size(); ++i) {
      const Part& p = parts[i];
      W[i] = need(p.prefix + ".weight");
      if (!W[i]) return VELLA_E_INVALID;
      S[i] = v.get(p.prefix + ".scales");
      B[i] = v.get(p.prefix + ".biases");
      int qb = 0;
      if (S[i]) {
        if (conv || !B[i] || W[i]->dtype != VELLA_ST_U32 || W[i]->shape.size() != 2 || W[i]->shape[0] != p.rows ||
            (W[i]->shape[1] * 32 != K * 4 && W[i]->shape[1] * 32 != K * 8))
          return fail(VELLA_E_INVALID, "checkpoint: '%s.weight' is not MLX-affine [%lld, %lld*bits/32] u32",
                      p.prefix.c_str(), (long long)p.rows, (long long)K);
        qb = (int)(W[i]->shape[1] * 32 / K);
        if (K % 64 || !is_float(*S[i]) || !is_float(*B[i]) || !shape_is(S[i], {p.rows, K / 64}) ||
            !shape_is(B[i], {p.rows, K / 64}))
          return fail(VELLA_E_UNSUPPORTED, "checkpoint: '%s' scales/biases are not [%lld, %lld] (group 64)",
                      p.prefix.c_str(), (long long)p.rows, (long long)(K / 64));
      } else {
        const int64_t C = K / 3;
        const bool ok = is_float(*W[i]) && (conv ? shape_is(W[i], {p.rows, v.hf ? C : 3, v.hf ? 3 : C})
                                                  : shape_is(W[i], {p.rows, K}));
        if (!ok)
          return fail(VELLA_E_INVALID, "checkpoint: '%s.weight' must be a float %s", p.prefix.c_str(),
                      conv ? "Conv1d weight (kernel 3)" : "matrix of the handle's shape");
      }
      if (qbits >= 0 && qbits != qb)
        return fail(VELLA_E_UNSUPPORTED, "checkpoint: '%s' mixes float and quantized parts", dname.c_str());
      qbits = qb;
      if (with_bias && p.bias) {
        Bias[i] = need(p.prefix + ".bias");
        if (!Bias[i]) return VELLA_E_INVALID;
        if (!is_float(*Bias[i]) || !shape_is(Bias[i], {p.rows}))
          return fail(VELLA_E_INVALID, "checkpoint: '%s.bias' must be a float [%lld]", p.prefix.c_str(),
                      (long long)p.rows);
      }
    }
    if (qbits > 0 && bits > 0 && qbits != bits)
      return fail(VELLA_E_UNSUPPORTED, "checkpoint: '%s' is %d-bit, the handle %d-bit", dname.c_str(), qbits,
                  bits);
    if (with_bias) {
      void* d = nullptr;
      int rc = dest(dname + ".bias", layer, (size_t)N * 2, &d);
      if (rc) return rc;
      if (w) {
        std::vector<uint16_t> h((size_t)N, act_bits(0.0f, act));
        int64_t r0 = 0;
        for (size_t i = 0; i < parts.size(); ++i) {
          if (Bias[i])
            for (int64_t r = 0; r < parts[i].rows; ++r) h[(size_t)(r0 + r)] = act_bits(elem_f(*Bias[i], (size_t)r), act);
          r0 += parts[i].rows;
        }
        if ((rc = put(d, h.data(), h.size() * 2))) return rc;
      }
    }
    if (bits > 0 && qbits > 0) return copy_packed(dname, layer, parts, W, S, B, N, K, bits);
    if (bits > 0) return quantize(dname, layer, parts, W, N, K, bits);
    if (qbits == 0 && fake_bits > 0 && !conv && kpad == K) return fake_quant(dname, layer, parts, W, N, K);
    return dense(dname, layer, parts, W, S, B, N, K, kpad, conv, qbits);
  }

  // value (r, k) of part i as float: a float matrix or Conv1d weight, or MLX-affine s*q + b
  float part_val(const StEntry* W, const StEntry* S, const StEntry* B, int qb, int64_t r, int64_t k, int64_t K,
                 bool conv) const {
    if (qb > 0) {
      const int per = 32 / qb;
      uint32_t word;
      std::memcpy(&word, W->data + ((size_t)r * (size_t)(K / per) + (size_t)(k / per)) * 4, 4);
      const uint32_t q = (word >> ((k % per) * qb)) & ((1u << qb) - 1u);
      const size_t g = (size_t)r * (size_t)(K / 64) + (size_t)(k / 64);
      float x = elem_f(*S, g) * (float)q;  // scale * q, then + bias: two roundings, as the kernels
      x = x + elem_f(*B, g);
      return x;
    }
    if (conv) {
      const int64_t C = K / 3, j = k / C, ch = k % C;
      return elem_f(*W, v.hf ? (size_t)((r * C + ch) * 3 + j) : (size_t)((r * 3 + j) * C + ch));
    }
    return elem_f(*W, (size_t)(r * K + k));
  }

  int dense(const std::string& dname, int layer, const std::vector<Part>& parts, const std::vector<const StEntry*>& W,
            const std::vector<const StEntry*>& S, const std::vector<const StEntry*>& B, int64_t N, int64_t K,
            int64_t kpad, bool conv, int qb) {
    void* d = nullptr;
    int rc = dest(dname + ".w", layer, (size_t)N * kpad * 2, &d);
    if (rc || !w) return rc;
    std::vector<uint16_t> h((size_t)N * kpad, act_bits(0.0f, act));
    int64_t r0 = 0;
    for (size_t i = 0; i < parts.size(); ++i) {
      for (int64_t r = 0; r < parts[i].rows; ++r)
        for (int64_t k = 0; k < K; ++k)
          h[(size_t)((r0 + r) * kpad + k)] = act_bits(part_val(W[i], S[i], B[i], qb, r, k, K, conv), act);
      r0 += parts[i].rows;
    }
    return put(d, h.data(), h.size() * 2);
  }

  int copy_packed(const std::string& dname, int layer, const std::vector<Part>& parts,
                  const std::vector<const StEntry*>& W, const std::vector<const StEntry*>& S,
                  const std::vector<const StEntry*>& B, int64_t N, int64_t K, int bits) {
    void *dw = nullptr, *ds = nullptr, *db = nullptr;
    const size_t wb = (size_t)N * (size_t)(K * bits / 32) * 4, sb = (size_t)N * (size_t)(K / 64) * 2;
    int rc;
    if ((rc = dest(dname + ".w", layer, wb, &dw)) || (rc = dest(dname + ".s", layer, sb, &ds)) ||
        (rc = dest(dname + ".b", layer, sb, &db)) || !w)
      return rc;
    std::vector<uint8_t> hw(wb);
    std::vector<uint16_t> hs((size_t)N * (size_t)(K / 64)), hb(hs.size());
    size_t ow = 0, og = 0;
    for (size_t i = 0; i < parts.size(); ++i) {
      std::memcpy(hw.data() + ow, W[i]->data, W[i]->bytes);
      ow += W[i]->bytes;
      const size_t ng = (size_t)parts[i].rows * (size_t)(K / 64);
      for (size_t g = 0; g < ng; ++g) {
        hs[og + g] = act_bits(elem_f(*S[i], g), act);
        hb[og + g] = act_bits(elem_f(*B[i], g), act);
      }
      og += ng;
    }
    if ((rc = put(dw, hw.data(), wb)) || (rc = put(ds, hs.data(), sb))) return rc;
    return put(db, hb.data(), sb);
  }

  // derived precision: the float rows quantized on the device straight into the handle's
  // packed weight, scales and biases
  int quantize(const std::string& dname, int layer, const std::vector<Part>& parts,
               const std::vector<const StEntry*>& W, int64_t N, int64_t K, int bits) {
    void *dw = nullptr, *ds = nullptr, *db = nullptr;
    const size_t wb = (size_t)N * (size_t)(K * bits / 32) * 4, sb = (size_t)N * (size_t)(K / 64) * 2;
    int rc;
    if ((rc = dest(dname + ".w", layer, wb, &dw)) || (rc = dest(dname + ".s", layer, sb, &ds)) ||
        (rc = dest(dname + ".b", layer, sb, &db)) || !w)
      return rc;
    return quantize_into(parts, W, N, K, bits, dw, ds, db);
  }

  // the dense weight of a derived precision's Linear: MLX-affine at fake_bits, dequantized
  int fake_quant(const std::string& dname, int layer, const std::vector<Part>& parts,
                 const std::vector<const StEntry*>& W, int64_t N, int64_t K) {
    void* d = nullptr;
    int rc = dest(dname + ".w", layer, (size_t)(N * K) * 2, &d);
    if (rc || !w) return rc;
    const int bits = fake_bits;
    const size_t wb = (size_t)N * (size_t)(K * bits / 32) * 4, sb = (size_t)N * (size_t)(K / 64) * 2;
    void* tmp = nullptr;
    VELLA_CUDA_TRY(cudaMalloc(&tmp, wb + 2 * sb));
    char* t = static_cast<char*>(tmp);
    rc = quantize_into(parts, W, N, K, bits, t, t + wb, t + wb + sb);
    cudaError_t e = cudaSuccess;
    if (!rc) {
      const int64_t n = N * K;
      const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
      if (act == VELLA_F16)
        dequant_rows_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<__half*>(d), reinterpret_cast<uint32_t*>(t),
                                                               reinterpret_cast<__half*>(t + wb),
                                                               reinterpret_cast<__half*>(t + wb + sb), K, bits, n);
      else
        dequant_rows_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
            static_cast<__nv_bfloat16*>(d), reinterpret_cast<uint32_t*>(t),
            reinterpret_cast<__nv_bfloat16*>(t + wb), reinterpret_cast<__nv_bfloat16*>(t + wb + sb), K, bits, n);
      e = cudaGetLastError();
      if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    }
    cudaFree(tmp);
    if (rc) return rc;
    if (e != cudaSuccess) return vella::cuda_fail(e, "checkpoint load: dequantize");
    return VELLA_OK;
  }

  // the float rows (in the source dtype when every part shares it, else fp32) quantized on
  // the device into packed weight, scales and biases
  int quantize_into(const std::vector<Part>& parts, const std::vector<const StEntry*>& W, int64_t N, int64_t K,
                    int bits, void* dw, void* ds, void* db) {
    int rc = VELLA_OK;
    int src = W[0]->dtype;
    for (const StEntry* e : W)
      if (e->dtype != src) src = VELLA_ST_F32;
    const size_t es = src == VELLA_ST_F32 ? 4 : 2;
    std::vector<uint8_t> h((size_t)N * (size_t)K * es);
    size_t o = 0;
    for (size_t i = 0; i < parts.size(); ++i) {
      if (W[i]->dtype == src) {
        std::memcpy(h.data() + o, W[i]->data, W[i]->bytes);
        o += W[i]->bytes;
      } else {
        const size_t n = W[i]->numel();
        for (size_t j = 0; j < n; ++j) {
          const float f = elem_f(*W[i], j);
          std::memcpy(h.data() + o + j * 4, &f, 4);
        }
        o += n * 4;
      }
    }
    void* tmp = nullptr;
    VELLA_CUDA_TRY(cudaMalloc(&tmp, h.size()));
    vella_qgemm_desc qd{};
    qd.m = 1;
    qd.n = (int32_t)N;
    qd.k = (int32_t)K;
    qd.bits = bits;
    qd.group_size = 64;
    qd.dtype = act;
    cudaError_t e = cudaMemcpyAsync(tmp, h.data(), h.size(), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) {
      rc = vella_quantize(&qd, src, tmp, dw, ds, db, stream);
      e = cudaStreamSynchronize(stream);
    }
    cudaFree(tmp);
    if (rc) return rc;
    if (e != cudaSuccess) return vella::cuda_fail(e, "checkpoint load: quantize");
    return VELLA_OK;
  }
};


int whisper_tensors(Loader& L, const vella_whisper_cfg& c) {
  const int64_t d = c.d_model, F = c.ffn;
  const int bits = c.bits;
  const int64_t kp1 = (3 * c.n_mels + 63) / 64 * 64;
  int rc;
  const std::string E = "model.encoder.", D = "model.decoder.";
  if ((rc = L.linear("conv1", -1, {{E + "conv1", d, true}}, 3 * c.n_mels, 0, kp1, true, true))) return rc;
  if ((rc = L.linear("conv2", -1, {{E + "conv2", d, true}}, 3 * d, 0, 3 * d, true, true))) return rc;
  if ((rc = L.table("enc_pos", E + "embed_positions.weight", c.n_audio, d, true))) return rc;
  if ((rc = L.vec("enc_ln.weight", -1, E + "layer_norm.weight", d)) || (rc = L.vec("enc_ln.bias", -1, E + "layer_norm.bias", d)))
    return rc;
  // a derived precision (float checkpoint, int handle) quantizes the encoder Linears too, as the
  // reference's does; an already-quantized checkpoint's float tensors stay float
  L.fake_bits = L.v.quantized ? 0 : bits;
  for (int l = 0; l < c.enc_layers; ++l) {
    const std::string p = E + "layers." + std::to_string(l) + ".";
    if ((rc = L.vec("enc.ln1.weight", l, p + "self_attn_layer_norm.weight", d)) ||
        (rc = L.vec("enc.ln1.bias", l, p + "self_attn_layer_norm.bias", d)) ||
        (rc = L.vec("enc.ln2.weight", l, p + "final_layer_norm.weight", d)) ||
        (rc = L.vec("enc.ln2.bias", l, p + "final_layer_norm.bias", d)))
      return rc;
    if ((rc = L.linear("enc.qkv", l,
                     {{p + "self_attn.q_proj", d, true}, {p + "self_attn.k_proj", d, false},
                      {p + "self_attn.v_proj", d, true}},
                     d, 0, d, false, true)) ||
        (rc = L.linear("enc.o", l, {{p + "self_attn.out_proj", d, true}}, d, 0, d, false, true)) ||
        (rc = L.linear("enc.fc1", l, {{p + "fc1", F, true}}, d, 0, d, false, true)) ||
        (rc = L.linear("enc.fc2", l, {{p + "fc2", d, true}}, F, 0, F, false, true)))
      return rc;
  }
  L.fake_bits = 0;
  if ((rc = L.linear("embed", -1, {{D + "embed_tokens", c.vocab, false}}, d, bits, d, false, false))) return rc;
  if ((rc = L.table("dec_pos", D + "embed_positions.weight", c.max_target, d, false))) return rc;
  if ((rc = L.vec("dec_ln.weight", -1, D + "layer_norm.weight", d)) || (rc = L.vec("dec_ln.bias", -1, D + "layer_norm.bias", d)))
    return rc;
  for (int l = 0; l < c.dec_layers; ++l) {
    const std::string p = D + "layers." + std::to_string(l) + ".";
    static const std::pair<const char*, const char*> norms[] = {
        {"dec.ln1", "self_attn_layer_norm"}, {"dec.ln2", "encoder_attn_layer_norm"}, {"dec.ln3", "final_layer_norm"}};
    for (const auto& nm : norms)
      if ((rc = L.vec(std::string(nm.first) + ".weight", l, p + nm.second + ".weight", d)) ||
          (rc = L.vec(std::string(nm.first) + ".bias", l, p + nm.second + ".bias", d)))
        return rc;
    if ((rc = L.linear("dec.qkv", l,
                     {{p + "self_attn.q_proj", d, true}, {p + "self_attn.k_proj", d, false},
                      {p + "self_attn.v_proj", d, true}},
                     d, bits, d, false, true)) ||
        (rc = L.linear("dec.o", l, {{p + "self_attn.out_proj", d, true}}, d, bits, d, false, true)) ||
        (rc = L.linear("dec.cq", l, {{p + "encoder_attn.q_proj", d, true}}, d, bits, d, false, true)) ||
        (rc = L.linear("dec.ckv", l, {{p + "encoder_attn.k_proj", d, false}, {p + "encoder_attn.v_proj", d, true}}, d,
                     bits, d, false, true)) ||
        (rc = L.linear("dec.co", l, {{p + "encoder_attn.out_proj", d, true}}, d, bits, d, false, true)) ||
        (rc = L.linear("dec.fc1", l, {{p + "fc1", F, true}}, d, bits, d, false, true)) ||
        (rc = L.linear("dec.fc2", l, {{p + "fc2", d, true}}, F, bits, F, false, true)))
      return rc;
  }
  return VELLA_OK;
}

// Qwen3-style decoder (Qwen3ASRTextDecoder.swift:17-214; keys as Qwen3ASRModel.sanitize
// leaves them, Qwen3ASRModel.swift:682-708: a "thinker." prefix stripped):
// model.embed_tokens, model.norm, lm_head (absent when tied to the embedding), and per layer
// input_layernorm, post_attention_layernorm, self_attn.{q,k,v,o}_proj, self_attn.{q,k}_norm,
// mlp.{gate,up,down}_proj, none with a bias.
KeyView model_view(const vella_st* st) {
  KeyView v;
  for (const StEntry& e : st->entries) {
    const std::string k = starts(e.name, "thinker.") ? e.name.substr(8) : e.name;
    v.by[k] = &e;
  }
  return v;
}

int model_tensors(Loader& L, const vella_model_cfg& c) {
  const int64_t d = c.d_model, F = c.ffn, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads;
  const int bits = c.bits;
  int rc;
  if ((rc = L.linear("embed", -1, {{"model.embed_tokens", c.vocab, false}}, d, 0, d, false, false)))
    return rc;
  if ((rc = L.vec("final_norm", -1, "model.norm.weight", d))) return rc;
  // lm_head, or the embedding when the checkpoint ties them (no lm_head.weight)
  const char* head = L.v.get("lm_head.weight") ? "lm_head" : "model.embed_tokens";
  if ((rc = L.linear("lm_head", -1, {{head, c.vocab, false}}, d, bits, d, false, false))) return rc;
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    if ((rc = L.vec("attn_norm", l, p + "input_layernorm.weight", d)) ||
        (rc = L.vec("mlp_norm", l, p + "post_attention_layernorm.weight", d)))
      return rc;
    if (c.qk_norm && ((rc = L.vec("q_norm", l, p + "self_attn.q_norm.weight", hd)) ||
                      (rc = L.vec("k_norm", l, p + "self_attn.k_norm.weight", hd))))
      return rc;
    if ((rc = L.linear("qkv", l,
                       {{p + "self_attn.q_proj", H * hd, false}, {p + "self_attn.k_proj", KV * hd, false},
                        {p + "self_attn.v_proj", KV * hd, false}},
                       d, bits, d, false, false)) ||
        (rc = L.linear("o", l, {{p + "self_attn.o_proj", d, false}}, H * hd, bits, H * hd, false, false)) ||
        (rc = L.linear("gate", l, {{p + "mlp.gate_proj", F, false}}, d, bits, d, false, false)) ||
        (rc = L.linear("up", l, {{p + "mlp.up_proj", F, false}}, d, bits, d, false, false)) ||
        (rc = L.linear("down", l, {{p + "mlp.down_proj", d, false}}, F, bits, F, false, false)))
      return rc;
  }
  return VELLA_OK;
}

// Nemotron-H (NemotronTranscribeKeys.map, NemotronTranscribeText.swift:369-397; NTMTP.nvidiaKeys,
// NemotronTranscribeDecoder.swift:608-626): NVIDIA's NeMo keys (llm.model.*, llm.mtp.*) or the
// MLX module tree (llm.backbone.*, mtp.*), onto backbone.* / lm_head / mtp.* names; NeMo's stacked
// experts are [E][in][out] (marked transposed); a depthwise conv weight is [C][K] in memory in
// every layout.
KeyView nh_view(const vella_st* st) {
  KeyView v;
  static const std::pair<const char*, const char*> mtp_keys[] = {
      {"llm.mtp.layers.0.eh_proj.weight", "mtp.eh_proj.weight"},
      {"llm.mtp.layers.0.enorm.weight", "mtp.enorm.weight"},
      {"llm.mtp.layers.0.hnorm.weight", "mtp.hnorm.weight"},
      {"llm.mtp.layers.0.norm.weight", "mtp.attn_norm.weight"},
      {"llm.mtp.layers.0.mixer.q_proj.weight", "mtp.attn.q_proj.weight"},
      {"llm.mtp.layers.0.mixer.k_proj.weight", "mtp.attn.k_proj.weight"},
      {"llm.mtp.layers.0.mixer.v_proj.weight", "mtp.attn.v_proj.weight"},
      {"llm.mtp.layers.0.mixer.o_proj.weight", "mtp.attn.o_proj.weight"},
      {"llm.mtp.layers.1.norm.weight", "mtp.moe_norm.weight"},
      {"llm.mtp.layers.1.mixer.gate.weight", "mtp.moe.gate.weight"},
      {"llm.mtp.layers.1.mixer.gate.e_score_correction_bias", "mtp.moe.gate.e_score_correction_bias"},
      {"llm.mtp.layers.1.mixer.shared_experts.up_proj.weight", "mtp.moe.shared_experts.up_proj.weight"},
      {"llm.mtp.layers.1.mixer.shared_experts.down_proj.weight", "mtp.moe.shared_experts.down_proj.weight"},
      {"llm.mtp.layers.1.mixer.experts.gate_and_up_projs", "mtp.moe.switch_mlp.fc1.weight"},
      {"llm.mtp.layers.1.mixer.experts.down_projs", "mtp.moe.switch_mlp.fc2.weight"},
      {"llm.mtp.layers.1.final_layernorm.weight", "mtp.final_norm.weight"}};
  auto replace_all = [](std::string k, const char* from, const char* to) {
    for (size_t at = k.find(from); at != std::string::npos; at = k.find(from, at + std::strlen(to)))
      k.replace(at, std::strlen(from), to);
    return k;
  };
  for (const StEntry& e : st->entries) {
    std::string k = e.name;
    bool tr = false, known = false;
    for (const auto& mk : mtp_keys)
      if (k == mk.first) {
        tr = starts(k, "llm.mtp.") && k.size() > 6 && k.compare(k.size() - 6, 6, "_projs") == 0;
        k = mk.second;
        known = true;
      }
    if (!known) {
      if (starts(k, "llm.mtp.") || starts(k, "ctc_timestamp.") || k.find("._extra_state") != std::string::npos) continue;
      if (starts(k, "llm.model.")) {
        k = replace_all(k, "llm.model.embed_tokens.", "backbone.embeddings.");
        k = replace_all(k, "llm.model.norm.", "backbone.norm_f.");
        k = replace_all(k, "llm.model.layers.", "backbone.layers.");
        k = replace_all(k, "._fp32_params.", ".");
        if (k.find(".experts.gate_and_up_projs") != std::string::npos) {
          k = replace_all(k, ".experts.gate_and_up_projs", ".switch_mlp.fc1.weight");
          tr = true;
        } else if (k.find(".experts.down_projs") != std::string::npos) {
          k = replace_all(k, ".experts.down_projs", ".switch_mlp.fc2.weight");
          tr = true;
        }
      } else if (starts(k, "llm.")) {
        k = k.substr(4);  // llm.backbone.* / llm.lm_head.*
      }
    }
    v.by[k] = &e;
    if (tr) v.transposed[k] = true;
    if (k.size() > 7 && k.compare(k.size() - 7, 7, ".scales") == 0) v.quantized = true;
  }
  return v;
}

int nh_attention_tensors(Loader& L, const vella_nh_cfg& c, const std::string& p, const std::string& dq, int layer) {
  const int64_t d = c.hidden, hd = c.head_dim;
  int rc;
  if ((rc = L.linear(dq + "qkv", layer,
                     {{p + "q_proj", c.heads * hd, false}, {p + "k_proj", c.kv_heads * hd, false},
                      {p + "v_proj", c.kv_heads * hd, false}},
                     d, c.bits, d, false, false)))
    return rc;
  return L.linear(dq + "o", layer, {{p + "o_proj", d, false}}, c.heads * hd, c.bits, c.heads * hd, false, false);
}

int nh_moe_tensors(Loader& L, const vella_nh_cfg& c, const std::string& p, const std::string& dq, int layer) {
  const int64_t d = c.hidden;
  int rc;
  if ((rc = L.f32(dq + "router", layer, p + "gate.weight", (int64_t)c.experts * d)) ||
      (rc = L.f32(dq + "router_bias", layer, p + "gate.e_score_correction_bias", c.experts)) ||
      (rc = L.experts(dq + "fc1", layer, p + "switch_mlp.fc1", c.experts, c.moe_inter, d, c.bits)) ||
      (rc = L.experts(dq + "fc2", layer, p + "switch_mlp.fc2", c.experts, d, c.moe_inter, c.bits)) ||
      (rc = L.linear(dq + "shared_up", layer, {{p + "shared_experts.up_proj", c.shared_inter, false}}, d, c.bits, d,
                     false, false)))
    return rc;
  return L.linear(dq + "shared_down", layer, {{p + "shared_experts.down_proj", d, false}}, c.shared_inter, c.bits,
                  c.shared_inter, false, false);
}

int nh_tensors(Loader& L, const vella_nh_cfg& c) {
  const int64_t d = c.hidden, I = (int64_t)c.m_heads * c.m_head_dim;
  const int64_t conv_dim = I + 2LL * c.groups * c.state_dim, in_w = I + conv_dim + c.m_heads;
  int rc;
  if ((rc = L.linear("embed", -1, {{"backbone.embeddings", c.vocab, false}}, d, 0, d, false, false)) ||
      (rc = L.vec("norm_f", -1, "backbone.norm_f.weight", d)) ||
      (rc = L.linear("lm_head", -1, {{"lm_head", c.vocab, false}}, d, c.bits, d, false, false)))
    return rc;
  const int Lcount = (int)strnlen(c.pattern, sizeof(c.pattern));
  for (int l = 0; l < Lcount; ++l) {
    const std::string p = "backbone.layers." + std::to_string(l) + ".";
    if ((rc = L.vec("norm", l, p + "norm.weight", d))) return rc;
    const std::string mx = p + "mixer.";
    if (c.pattern[l] == 'M') {
      if ((rc = L.linear("in_proj", l, {{mx + "in_proj", in_w, false}}, d, c.bits, d, false, false)) ||
          (rc = L.linear("out_proj", l, {{mx + "out_proj", d, false}}, I, c.bits, I, false, false)) ||
          (rc = L.flat("conv_w", l, mx + "conv1d.weight", conv_dim * c.conv_kernel)) ||
          (rc = L.flat("conv_b", l, mx + "conv1d.bias", conv_dim)) ||
          (rc = L.flat("gnorm", l, mx + "norm.weight", I)) ||
          (rc = L.f32("a_log", l, mx + "A_log", c.m_heads)) || (rc = L.f32("dt_bias", l, mx + "dt_bias", c.m_heads)) ||
          (rc = L.f32("D", l, mx + "D", c.m_heads)))
        return rc;
    } else if (c.pattern[l] == '*') {
      if ((rc = nh_attention_tensors(L, c, mx, "", l))) return rc;
    } else {
      if ((rc = nh_moe_tensors(L, c, mx, "", l))) return rc;
    }
  }
  if (c.mtp) {
    if ((rc = L.linear("mtp.eh_proj", -1, {{"mtp.eh_proj", d, false}}, 2 * d, c.bits, 2 * d, false, false)) ||
        (rc = L.vec("mtp.enorm", -1, "mtp.enorm.weight", d)) || (rc = L.vec("mtp.hnorm", -1, "mtp.hnorm.weight", d)) ||
        (rc = L.vec("mtp.attn_norm", -1, "mtp.attn_norm.weight", d)) ||
        (rc = L.vec("mtp.moe_norm", -1, "mtp.moe_norm.weight", d)) ||
        (rc = L.vec("mtp.final_norm", -1, "mtp.final_norm.weight", d)) ||
        (rc = nh_attention_tensors(L, c, "mtp.attn.", "mtp.", -1)) || (rc = nh_moe_tensors(L, c, "mtp.moe.", "mtp.", -1)))
      return rc;
  }
  return VELLA_OK;
}

// Checks every key and shape, then fills the handle on a private stream of the device that
// holds `probe` (a device pointer of the handle).
int check_then_fill(const KeyView& v, int act, const TensorFn& tensor, const void* probe,
                    const std::function<int(Loader&)>& walk) {
  Loader chk{TensorFn(), v, act};
  int rc = walk(chk);
  if (rc) return rc;  // a failed check leaves the handle as it was
  cudaPointerAttributes at{};
  VELLA_CUDA_TRY(cudaPointerGetAttributes(&at, probe));
  VELLA_CUDA_TRY(cudaSetDevice(at.device));
  Loader L{tensor, v, act};
  L.w = true;
  VELLA_CUDA_TRY(cudaStreamCreateWithFlags(&L.stream, cudaStreamNonBlocking));
  rc = walk(L);
  cudaStreamDestroy(L.stream);
  return rc;
}

}  // namespace

extern "C" {

int vella_st_open(const char* const* paths, int32_t n_paths, vella_st** out) {
  if (!paths || n_paths < 1 || !out) return fail(VELLA_E_INVALID, "vella_st_open: no files");
  *out = nullptr;
  auto st = std::make_unique<vella_st>();
  for (int i = 0; i < n_paths; ++i) {
    if (!paths[i]) return fail(VELLA_E_INVALID, "vella_st_open: NULL path");
    const int rc = st_add_file(st.get(), paths[i]);
    if (rc) return rc;
  }
  *out = st.release();
  return VELLA_OK;
}

int vella_st_close(vella_st* st) {
  delete st;
  return VELLA_OK;
}

int vella_st_count(const vella_st* st, int32_t* n) {
  if (!st || !n) return fail(VELLA_E_INVALID, "vella_st_count: NULL argument");
  *n = (int32_t)st->entries.size();
  return VELLA_OK;
}

int vella_st_find(const vella_st* st, const char* name, int32_t* index) {
  if (!st || !name || !index) return fail(VELLA_E_INVALID, "vella_st_find: NULL argument");
  const auto it = st->index.find(name);
  *index = it == st->index.end() ? -1 : it->second;
  return VELLA_OK;
}

int vella_st_info(const vella_st* st, int32_t index, const char** name, int32_t* dtype, int32_t* ndim,
                  int64_t* shape, const void** data, size_t* bytes) {
  if (!st || index < 0 || index >= (int32_t)st->entries.size())
    return fail(VELLA_E_INVALID, "vella_st_info: index %d out of range", index);
  const StEntry& e = st->entries[(size_t)index];
  if (name) *name = e.name.c_str();
  if (dtype) *dtype = e.dtype;
  if (ndim) *ndim = (int32_t)e.shape.size();
  if (shape)
    for (size_t i = 0; i < e.shape.size(); ++i) shape[i] = e.shape[i];
  if (data) *data = e.data;
  if (bytes) *bytes = e.bytes;
  return VELLA_OK;
}

int vella_whisper_check_checkpoint(const vella_st* st, const vella_whisper_cfg* cfg) {
  if (!st || !cfg) return fail(VELLA_E_INVALID, "vella_whisper_check_checkpoint: NULL argument");
  const KeyView v = whisper_view(st);
  Loader L{TensorFn(), v, cfg->dtype};
  return whisper_tensors(L, *cfg);
}

int vella_whisper_load(vella_whisper* w, const vella_st* st) {
  if (!w || !st) return fail(VELLA_E_INVALID, "vella_whisper_load: NULL argument");
  vella_whisper_cfg c{};
  int rc = vella_whisper_get_cfg(w, &c);
  if (rc) return rc;
  void* probe = nullptr;
  size_t b = 0;
  if ((rc = vella_whisper_tensor(w, "dec_pos", -1, &probe, &b))) return rc;
  const KeyView v = whisper_view(st);
  const TensorFn fn = [w](const char* n, int l, void** p, size_t* sz) { return vella_whisper_tensor(w, n, l, p, sz); };
  rc = check_then_fill(v, c.dtype, fn, probe, [&c](Loader& L) { return whisper_tensors(L, c); });
  return rc ? rc : vella::whisper_weights_loaded(w);
}

int vella_nh_check_checkpoint(const vella_st* st, const vella_nh_cfg* cfg) {
  if (!st || !cfg) return fail(VELLA_E_INVALID, "vella_nh_check_checkpoint: NULL argument");
  const KeyView v = nh_view(st);
  Loader L{TensorFn(), v, cfg->dtype};
  return nh_tensors(L, *cfg);
}

int vella_nh_load(vella_nh* m, const vella_st* st) {
  if (!m || !st) return fail(VELLA_E_INVALID, "vella_nh_load: NULL argument");
  vella_nh_cfg cfg{};
  int rc = vella_nh_get_cfg(m, &cfg);
  if (rc) return rc;
  void* probe = nullptr;
  size_t b = 0;
  if ((rc = vella_nh_tensor(m, "norm_f", -1, &probe, &b))) return rc;
  const KeyView v = nh_view(st);
  // the dense embedding is the tensor "embed" (the loader asks for "embed.w")
  const TensorFn fn = [m](const char* n, int l, void** p, size_t* sz) {
    return vella_nh_tensor(m, std::strcmp(n, "embed.w") == 0 ? "embed" : n, l, p, sz);
  };
  const vella_nh_cfg c = cfg;
  return check_then_fill(v, c.dtype, fn, probe, [&c](Loader& L) { return nh_tensors(L, c); });
}

int vella_model_check_checkpoint(const vella_st* st, const vella_model_cfg* cfg) {
  if (!st || !cfg) return fail(VELLA_E_INVALID, "vella_model_check_checkpoint: NULL argument");
  const KeyView v = model_view(st);
  Loader L{TensorFn(), v, cfg->dtype};
  return model_tensors(L, *cfg);
}

int vella_model_load(vella_model* m, const vella_st* st) {
  if (!m || !st) return fail(VELLA_E_INVALID, "vella_model_load: NULL argument");
  vella_model_cfg c{};
  int rc = vella_model_get_cfg(m, &c);
  if (rc) return rc;
  void* probe = nullptr;
  size_t b = 0;
  if ((rc = vella_model_tensor(m, "embed", -1, &probe, &b))) return rc;
  const KeyView v = model_view(st);
  // the dense embedding is the tensor "embed" (the loader asks for "embed.w")
  const TensorFn fn = [m](const char* n, int l, void** p, size_t* sz) {
    return vella_model_tensor(m, std::strcmp(n, "embed.w") == 0 ? "embed" : n, l, p, sz);
  };
  return check_then_fill(v, c.dtype, fn, probe, [&c](Loader& L) { return model_tensors(L, c); });
}

}  // extern "C"
