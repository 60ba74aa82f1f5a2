// voice.cu — Voice::save / Voice::load (tts/voice.rs:78-149): a stream's KV state in the
// safetensors layout of upstream Pocket TTS, read back into many streams of a state at once.
//
// File layout (one entry per layer i, the reference's names):
//   transformer.layers.{i}.self_attn/cache   [2, 1, len, kv_heads, head_dim]  keys, values
//   transformer.layers.{i}.self_attn/offset  i64 [1] = len (older files: the shape of
//                                            .../current_end, else the time axis)
//   transformer.layers.{i}.self_attn/pad     i64 [1] = 0 (padded, batched states are refused)
// safetensors: an 8-byte little-endian header length, a JSON header mapping each name to
// {dtype, shape, data_offsets}, then the data.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "engine.h"

namespace svl {
namespace {

// ---- a JSON reader for safetensors headers ------------------------------------------------

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;
};

struct JsonParser {
  const char* p;
  const char* e;
  [[noreturn]] void fail(const std::string& what) { throw Error(SVL_ERR_INVALID_INPUT, "voice file header: " + what); }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      p++;
      return true;
    }
    return false;
  }
  std::string string() {
    if (!eat('"')) fail("expected a string");
    std::string s;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) fail("bad escape");
        const char c = *p++;
        switch (c) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {
            if (e - p < 4) fail("bad escape");
            const unsigned code = (unsigned)std::stoul(std::string(p, p + 4), nullptr, 16);
            p += 4;
            if (code < 0x80) s += (char)code; else s += '?';  // names are ASCII
            break;
          }
          default: s += c;
        }
      } else {
        s += *p++;
      }
    }
    if (p >= e) fail("unterminated string");
    p++;
    return s;
  }
  Json value() {
    ws();
    if (p >= e) fail("truncated");
    Json j;
    if (*p == '{') {
      p++;
      j.kind = Json::OBJ;
      if (eat('}')) return j;
      do {
        std::string k = string();
        if (!eat(':')) fail("expected ':'");
        j.obj[k] = value();
      } while (eat(','));
      if (!eat('}')) fail("expected '}'");
    } else if (*p == '[') {
      p++;
      j.kind = Json::ARR;
      if (eat(']')) return j;
      do j.arr.push_back(value());
      while (eat(','));
      if (!eat(']')) fail("expected ']'");
    } else if (*p == '"') {
      j.kind = Json::STR;
      j.str = string();
    } else if (!strncmp(p, "true", 4) || !strncmp(p, "false", 5)) {
      j.kind = Json::BOOL;
      p += *p == 't' ? 4 : 5;
    } else if (!strncmp(p, "null", 4)) {
      p += 4;
    } else {
      char* end = nullptr;
      j.num = strtod(p, &end);
      if (end == p) fail("unexpected character");
      j.kind = Json::NUM;
      p = end;
    }
    return j;
  }
};

struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

struct StFile {
  std::vector<uint8_t> data;  // the data section
  std::map<std::string, StTensor> tensors;

  // Element i of tensor t as a double (f32 / f16 / bf16 / i64 / i32).
  double at(const StTensor& t, int64_t i) const {
    const uint8_t* b = data.data() + t.begin;
    if (t.dtype == "F32") { float f; memcpy(&f, b + 4 * i, 4); return f; }
    if (t.dtype == "I64") { int64_t v; memcpy(&v, b + 8 * i, 8); return (double)v; }
    if (t.dtype == "I32") { int32_t v; memcpy(&v, b + 4 * i, 4); return v; }
    if (t.dtype == "BF16") {
      uint16_t h; memcpy(&h, b + 2 * i, 2);
      uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f;
    }
    if (t.dtype == "F16") {
      uint16_t h; memcpy(&h, b + 2 * i, 2);
      const uint32_t sign = (h & 0x8000u) << 16, ex = (h >> 10) & 0x1f, man = h & 0x3ff;
      float f;
      if (ex == 0) f = std::ldexp((float)man, -24);
      else if (ex == 31) { uint32_t u = sign | 0x7f800000u | (man << 13); memcpy(&f, &u, 4); return f; }
      else f = std::ldexp((float)(man | 0x400), (int)ex - 25);
      return sign ? -f : f;
    }
    throw Error(SVL_ERR_INVALID_INPUT, "voice file: unsupported dtype " + t.dtype);
  }
};

size_t dtype_size(const std::string& d) {
  if (d == "F32" || d == "I32") return 4;
  if (d == "I64" || d == "F64") return 8;
  if (d == "F16" || d == "BF16" || d == "I16") return 2;
  if (d == "U8" || d == "I8" || d == "BOOL") return 1;
  return 0;
}

StFile read_safetensors(const char* path) {
  FILE* f = fopen(path, "rb");
  if (!f) throw Error(SVL_ERR_INVALID_INPUT, std::string("cannot open voice file ") + path);
  std::vector<uint8_t> all;
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) all.insert(all.end(), buf, buf + n);
  fclose(f);
  if (all.size() < 8) throw Error(SVL_ERR_INVALID_INPUT, "voice file: too short");
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; i--) hlen = hlen << 8 | all[i];
  if (hlen > all.size() - 8) throw Error(SVL_ERR_INVALID_INPUT, "voice file: bad header length");
  const char* h = reinterpret_cast<const char*>(all.data() + 8);
  JsonParser jp{h, h + hlen};
  Json root = jp.value();
  if (root.kind != Json::OBJ) throw Error(SVL_ERR_INVALID_INPUT, "voice file: header is not an object");
  StFile out;
  out.data.assign(all.begin() + 8 + hlen, all.end());
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    auto field = [&](const char* k) -> const Json& {
      auto it = t.obj.find(k);
      if (t.kind != Json::OBJ || it == t.obj.end())
        throw Error(SVL_ERR_INVALID_INPUT, "voice file: tensor " + kv.first + " lacks " + k);
      return it->second;
    };
    StTensor st;
    st.dtype = field("dtype").str;
    for (const Json& d : field("shape").arr) st.shape.push_back((int64_t)d.num);
    const Json& off = field("data_offsets");
    if (off.arr.size() != 2) throw Error(SVL_ERR_INVALID_INPUT, "voice file: bad data_offsets");
    st.begin = (int64_t)off.arr[0].num;
    st.end = (int64_t)off.arr[1].num;
    const size_t es = dtype_size(st.dtype);
    if (!es || st.begin < 0 || st.end > (int64_t)out.data.size() || st.end - st.begin != st.numel() * (int64_t)es)
      throw Error(SVL_ERR_INVALID_INPUT, "voice file: tensor " + kv.first + " has inconsistent offsets");
    out.tensors[kv.first] = st;
  }
  return out;
}

// ---- writing ----------------------------------------------------------------------------

struct OutTensor {
  std::string name, dtype;
  std::vector<int64_t> shape;
  std::vector<uint8_t> bytes;
};

void write_safetensors(const char* path, const std::vector<OutTensor>& ts) {
  std::string h = "{";
  int64_t off = 0;
  for (size_t i = 0; i < ts.size(); i++) {
    if (i) h += ",";
    h += "\"" + ts[i].name + "\":{\"dtype\":\"" + ts[i].dtype + "\",\"shape\":[";
    for (size_t d = 0; d < ts[i].shape.size(); d++) h += (d ? "," : "") + std::to_string(ts[i].shape[d]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + (int64_t)ts[i].bytes.size()) + "]}";
    off += (int64_t)ts[i].bytes.size();
  }
  h += "}";
  while (h.size() % 8) h += ' ';
  FILE* f = fopen(path, "wb");
  if (!f) throw Error(SVL_ERR_INVALID_INPUT, std::string("cannot write voice file ") + path);
  uint8_t len[8];
  uint64_t hl = h.size();
  for (int i = 0; i < 8; i++) len[i] = (uint8_t)(hl >> (8 * i));
  bool ok = fwrite(len, 1, 8, f) == 8 && fwrite(h.data(), 1, h.size(), f) == h.size();
  for (const OutTensor& t : ts) ok = ok && fwrite(t.bytes.data(), 1, t.bytes.size(), f) == t.bytes.size();
  ok = fclose(f) == 0 && ok;
  if (!ok) throw Error(SVL_ERR_INVALID_INPUT, std::string("cannot write voice file ") + path);
}

const char* kLayerPrefix = "transformer.layers.";

// ---- device import ------------------------------------------------------------------------

// kv [layer][2][kv_heads][len][head_dim] f32 (entries of positions 0 .. len-1) into the rings of
// streams[0 .. n): the last `keep` entries, entry j at slot j % cap (the ring holds position p
// at p % cap).
__global__ void voice_import_kernel(const float* kv, int layers, int kvh, int len, int hd, int keep,
                                    const int* streams, int n, void* k_ring, void* v_ring,
                                    int64_t layer_stride, int64_t stream_stride, int cap, int bf16) {
  const int64_t per_stream = (int64_t)layers * 2 * kvh * keep * hd;
  const int64_t total = per_stream * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    const int d = (int)(r % hd); r /= hd;
    const int j = (int)(r % keep) + (len - keep); r /= keep;
    const int h = (int)(r % kvh); r /= kvh;
    const int kv_i = (int)(r % 2); r /= 2;
    const int l = (int)(r % layers); r /= layers;
    const int s = streams[r];
    const float x = kv[((((int64_t)l * 2 + kv_i) * kvh + h) * len + j) * hd + d];
    const int64_t off = (int64_t)l * layer_stride + (int64_t)s * stream_stride + ((int64_t)h * cap + j % cap) * hd + d;
    void* ring = kv_i ? v_ring : k_ring;
    if (bf16)
      reinterpret_cast<__nv_bfloat16*>(ring)[off] = __float2bfloat16_rn(x);
    else
      reinterpret_cast<float*>(ring)[off] = x;
  }
}

}  // namespace

void voice_save(State& s, int stream, const char* path) {
  const auto& c = s.m->cfg;
  const int kvh = c.num_kv_heads, hd = c.head_dim;
  std::vector<OutTensor> ts;
  std::vector<float> k((size_t)kvh * s.cap * hd), v(k.size());
  for (int l = 0; l < c.num_layers; l++) {
    int len = 0;
    state_export(s, stream, l, k.data(), v.data(), &len);
    // [2, 1, len, kv_heads, head_dim]: the reference stacks k, v transposed to time-major.
    OutTensor cache;
    const std::string module = std::string(kLayerPrefix) + std::to_string(l) + ".self_attn";
    cache.name = module + "/cache";
    cache.dtype = "F32";
    cache.shape = {2, 1, len, kvh, hd};
    cache.bytes.resize((size_t)2 * len * kvh * hd * 4);
    float* dst = reinterpret_cast<float*>(cache.bytes.data());
    for (int which = 0; which < 2; which++) {
      const float* src = which ? v.data() : k.data();
      for (int t = 0; t < len; t++)
        for (int h = 0; h < kvh; h++)
          memcpy(dst + (((size_t)which * len + t) * kvh + h) * hd, src + ((size_t)h * len + t) * hd, (size_t)hd * 4);
    }
    OutTensor off, pad;
    off.name = module + "/offset";
    off.dtype = "I64";
    off.shape = {1};
    const int64_t len64 = len, zero = 0;
    off.bytes.assign(reinterpret_cast<const uint8_t*>(&len64), reinterpret_cast<const uint8_t*>(&len64) + 8);
    pad.name = module + "/pad";
    pad.dtype = "I64";
    pad.shape = {1};
    pad.bytes.assign(reinterpret_cast<const uint8_t*>(&zero), reinterpret_cast<const uint8_t*>(&zero) + 8);
    ts.push_back(std::move(cache));
    ts.push_back(std::move(off));
    ts.push_back(std::move(pad));
  }
  write_safetensors(path, ts);
}

void voice_load(State& s, const int* streams, int n, const char* path) {
  const auto& c = s.m->cfg;
  const int L = c.num_layers, kvh = c.num_kv_heads, hd = c.head_dim;
  StFile f = read_safetensors(path);
  // Every layer's cache, by index.
  std::vector<const StTensor*> caches(L, nullptr);
  std::vector<int64_t> lens(L, -1);
  const std::string suffix = ".self_attn/cache";
  for (auto& kv : f.tensors) {
    const std::string& name = kv.first;
    if (name.compare(0, strlen(kLayerPrefix), kLayerPrefix) || name.size() <= suffix.size() ||
        name.compare(name.size() - suffix.size(), suffix.size(), suffix))
      continue;
    const std::string idx = name.substr(strlen(kLayerPrefix), name.size() - strlen(kLayerPrefix) - suffix.size());
    if (idx.empty() || idx.find_first_not_of("0123456789") != std::string::npos)
      throw Error(SVL_ERR_INVALID_INPUT, "voice file: bad tensor name " + name);
    const int i = std::stoi(idx);
    if (i < 0 || i >= L) throw Error(SVL_ERR_INVALID_INPUT, "voice file: layer " + idx + " is not in the model");
    const StTensor& t = kv.second;
    if (t.shape.size() != 5 || t.shape[0] != 2 || t.shape[3] != kvh || t.shape[4] != hd)
      throw Error(SVL_ERR_INVALID_INPUT, "voice file: " + name + " is not [2, batch, time, kv_heads, head_dim] of this model");
    if (t.shape[1] != 1) throw Error(SVL_ERR_INVALID_INPUT, "voice file: batched voice states are not supported");
    const std::string module = name.substr(0, name.size() - strlen("/cache"));
    int64_t len = t.shape[2];
    auto off = f.tensors.find(module + "/offset");
    auto end = f.tensors.find(module + "/current_end");
    if (off != f.tensors.end() && off->second.numel() >= 1) len = (int64_t)f.at(off->second, 0);
    else if (end != f.tensors.end() && !end->second.shape.empty()) len = end->second.shape[0];
    auto pad = f.tensors.find(module + "/pad");
    if (pad != f.tensors.end())
      for (int64_t e = 0; e < pad->second.numel(); e++)
        if (f.at(pad->second, e) != 0)
          throw Error(SVL_ERR_INVALID_INPUT, "voice file: padded (batched) voice states are not supported");
    if (len < 0 || len > t.shape[2]) throw Error(SVL_ERR_INVALID_INPUT, "voice file: offset beyond the cache");
    caches[i] = &t;
    lens[i] = len;
  }
  for (int l = 0; l < L; l++)
    if (!caches[l]) throw Error(SVL_ERR_INVALID_INPUT, "voice file: no cache for layer " + std::to_string(l));
  const int64_t len = lens[0];
  for (int l = 1; l < L; l++)
    if (lens[l] != len) throw Error(SVL_ERR_INVALID_INPUT, "voice file: layers of different lengths");
  if (!s.windowed && len > s.cap) throw Error(SVL_ERR_INVALID_INPUT, "voice file: longer than the state's max_positions");
  if (s.ref_order && len > s.rope_positions)
    throw Error(SVL_ERR_UNSUPPORTED, "voice file: longer than the reference-order RoPE table");
  for (int i = 0; i < n; i++)
    if (streams[i] < 0 || streams[i] >= s.max_batch) throw Error(SVL_ERR_INVALID_INPUT, "stream index out of range");
  // [layer][2][kv_heads][len][head_dim] f32 on the host, then once to the device.
  std::vector<float> kv((size_t)L * 2 * kvh * len * hd);
  for (int l = 0; l < L; l++) {
    const StTensor& t = *caches[l];
    const int64_t T = t.shape[2];
    for (int which = 0; which < 2; which++)
      for (int64_t j = 0; j < len; j++)
        for (int h = 0; h < kvh; h++)
          for (int d = 0; d < hd; d++)
            kv[((((size_t)l * 2 + which) * kvh + h) * len + j) * hd + d] =
                (float)f.at(t, (((int64_t)which * T + j) * kvh + h) * hd + d);
  }
  const int keep = s.windowed ? (int)std::min<int64_t>(len, s.cap) : (int)len;
  check_cuda(cudaDeviceSynchronize(), "voice load");
  cudaStream_t st = s.m->stream;
  DevBuf d_kv, d_streams;
  if (keep > 0 && n > 0) {
    d_kv.alloc(kv.size() * 4);
    d_streams.alloc((size_t)n * 4);
    check_cuda(cudaMemcpyAsync(d_kv.p, kv.data(), kv.size() * 4, cudaMemcpyHostToDevice, st), "voice upload");
    check_cuda(cudaMemcpyAsync(d_streams.p, streams, (size_t)n * 4, cudaMemcpyHostToDevice, st), "voice upload");
    voice_import_kernel<<<1184, 256, 0, st>>>(d_kv.as<float>(), L, kvh, (int)len, hd, keep, d_streams.as<int>(), n,
                                              s.k_ring.p, s.v_ring.p, s.ring_layer_stride, s.ring_stream_stride,
                                              s.cap, s.kv_elt == 2);
    check_cuda(cudaGetLastError(), "voice import");
  }
  // TransformerState::from_layer_caches: the streams continue at position len.
  for (int i = 0; i < n; i++) s.hpos[streams[i]] = (int)len;
  check_cuda(cudaMemcpyAsync(s.pos.p, s.hpos.data(), (size_t)s.max_batch * 4, cudaMemcpyHostToDevice, st), "voice position");
  check_cuda(cudaStreamSynchronize(st), "voice load");
}

}  // namespace svl
