// engine.cu — weight loading, per-stream state and the step sequence of the LM.
#include "engine.h"
#include "gemv_common.cuh"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <string>

namespace svl {

void check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  cudaGetLastError();
  if (e == cudaErrorMemoryAllocation)
    throw Error(SVL_ERR_OOM, std::string(what) + ": " + cudaGetErrorString(e));
  throw Error(SVL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
  if (this != &o) {
    if (p) cudaFree(p);
    p = o.p;
    bytes = o.bytes;
    o.p = nullptr;
    o.bytes = 0;
  }
  return *this;
}
DevBuf::~DevBuf() {
  if (p) cudaFree(p);
}
void DevBuf::alloc(size_t n) {
  if (p) cudaFree(p);
  p = nullptr;
  bytes = 0;
  if (n == 0) return;
  check_cuda(cudaMalloc(&p, n), "cudaMalloc");
  bytes = n;
}
HostBuf::~HostBuf() {
  if (p) cudaFreeHost(p);
}
void HostBuf::alloc(size_t n) {
  if (p) cudaFreeHost(p);
  p = nullptr;
  check_cuda(cudaMallocHost(&p, n ? n : 16), "cudaMallocHost");
  bytes = n;
}

Model::~Model() {
  if (stream) cudaStreamDestroy(stream);
}

State::~State() {
  for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
}

namespace {

struct Loader {
  Model& m;
  const svl_tensor_view* t;
  int n;
  DevBuf staging;

  const svl_tensor_view* find(const std::string& name) const {
    for (int i = 0; i < n; i++)
      if (t[i].name && name == t[i].name) return &t[i];
    return nullptr;
  }
  const svl_tensor_view& need(const std::string& name, int64_t numel) const {
    const svl_tensor_view* v = find(name);
    if (!v) throw Error(SVL_ERR_CONFIG, "missing tensor " + name);
    if (v->numel != numel)
      throw Error(SVL_ERR_CONFIG, "tensor " + name + ": " + std::to_string(v->numel) +
                                      " elements, expected " + std::to_string(numel));
    if (!v->data) throw Error(SVL_ERR_CONFIG, "tensor " + name + " has no data");
    return *v;
  }
  bool bf16() const { return m.cfg.weight_dtype == SVL_DT_BF16; }

  // f32 vector on the device (rounded to bf16 values when the model runs in bf16, as the
  // reference's loader converts every tensor to the model dtype).
  DevBuf vec(const std::string& name, int64_t numel) {
    const svl_tensor_view& v = need(name, numel);
    DevBuf b;
    b.alloc(numel * 4);
    // Every transfer is ordered on the model's (non-blocking) stream: a plain cudaMemcpy from
    // pageable memory may return before its DMA lands, unordered with that stream's kernels.
    check_cuda(cudaMemcpyAsync(b.p, v.data, numel * 4, cudaMemcpyHostToDevice, m.stream), "upload");
    if (bf16()) launch_round_bf16_inplace(b.as<float>(), numel, m.stream);
    check_cuda(cudaStreamSynchronize(m.stream), "upload");
    m.weight_bytes += numel * 4;
    return b;
  }

  float* stage(const svl_tensor_view& v) {
    size_t bytes = v.numel * 4;
    if (staging.bytes < bytes) {
      check_cuda(cudaStreamSynchronize(m.stream), "upload");
      staging.alloc(bytes);
    }
    check_cuda(cudaMemcpyAsync(staging.p, v.data, bytes, cudaMemcpyHostToDevice, m.stream), "upload");
    return staging.as<float>();
  }

  // Linear::from_weight (nn/mod.rs:76-88): Q8_0 / Q4_1 when requested and k % 32 == 0, else
  // dense in the model dtype.
  void linear(Linear& L, const std::string& wname, const std::string& bname, int n_out, int k,
              bool quantizable, int interleave = 0) {
    const svl_tensor_view& v = need(wname, (int64_t)n_out * k);
    if (k % QBLK) throw Error(SVL_ERR_UNSUPPORTED, "linear " + wname + ": k % 32 != 0");
    int wt = W_F32;
    switch (m.cfg.weight_dtype) {
      case SVL_DT_BF16: wt = W_BF16; break;
      case SVL_DT_Q8_0: wt = quantizable ? W_Q8 : W_F32; break;
      case SVL_DT_Q4_1: wt = quantizable ? W_Q4 : W_F32; break;
      default: wt = W_F32;
    }
    L.n = n_out;
    L.k = k;
    L.wtype = wt;
    L.interleave = interleave;
    L.row_stride = packed_row_stride(wt, k);
    L.w.alloc(L.row_stride * n_out);
    // Zero first: the unused blocks of a partial last super-block stay zero.
    check_cuda(cudaMemsetAsync(L.w.p, 0, L.row_stride * n_out, m.stream), "memset");
    float* src = stage(v);
    launch_pack_linear(src, L.w.as<uint8_t>(), L.row_stride, n_out, k, wt, interleave, m.stream);
    check_cuda(cudaStreamSynchronize(m.stream), "pack weights");
    if (wt == W_BF16 && !make_gemm_operand(L.tc, L.w.p, n_out, k, L.row_stride, 128))
      throw Error(SVL_ERR_CUDA, "linear " + wname + ": cannot encode its TMA tensor map");
    if (!bname.empty()) L.bias = vec(bname, n_out);
    m.weight_bytes += L.row_stride * n_out;
  }

  void norm(Norm& N, const std::string& prefix, int d) {
    if (m.cfg.norm_kind == SVL_NORM_RMS) {
      N.kind = NORM_RMS;
      N.w = vec(prefix + ".alpha", d);
    } else {
      N.kind = NORM_LAYER;
      N.w = vec(prefix + ".weight", d);
      N.b = vec(prefix + ".bias", d);
    }
    N.eps = m.cfg.norm_eps;
  }

  void transformer(const std::string& pre) {
    const auto& c = m.cfg;
    const int d = c.d_model, qd = c.num_heads * c.head_dim, kvd = c.num_kv_heads * c.head_dim;
    m.layers.resize(c.num_layers);
    for (int l = 0; l < c.num_layers; l++) {
      Layer& L = m.layers[l];
      const std::string p = pre + "layers." + std::to_string(l) + ".";
      norm(L.norm1, p + "norm1", d);
      norm(L.norm2, p + "norm2", d);
      if (c.layer_scale) {
        L.ls1 = vec(p + "layer_scale_1.scale", d);
        L.ls2 = vec(p + "layer_scale_2.scale", d);
      }
      // Attention::new (nn/transformer.rs:300-316): in_proj_weight (moshi) or
      // in_proj.weight (Pocket TTS).
      std::string inw = p + "self_attn.in_proj_weight";
      if (!find(inw)) inw = p + "self_attn.in_proj.weight";
      linear(L.in_proj, inw, "", qd + 2 * kvd, d, true);
      linear(L.out_proj, p + "self_attn.out_proj.weight", "", d, qd, true);
      // FeedForwardLayer::new (nn/transformer.rs:418-436).
      if (c.ffn_kind == SVL_FFN_GATED_SILU) {
        linear(L.ff1, p + "gating.linear_in.weight", "", 2 * c.ffn_hidden, d, true, c.ffn_hidden);
        linear(L.ff2, p + "gating.linear_out.weight", "", d, c.ffn_hidden, true);
      } else {
        linear(L.ff1, p + "linear1.weight", "", c.ffn_hidden, d, true);
        linear(L.ff2, p + "linear2.weight", "", d, c.ffn_hidden, true);
      }
    }
    // RoPE inverse frequencies: computed in f64, stored f32 (nn/transformer.rs:114-118).
    const int half = c.head_dim / 2;
    std::vector<float> inv(half);
    for (int i = 0; i < half; i++)
      inv[i] = (float)std::exp(-std::log(c.max_period) * 2.0 * (double)i / (double)c.head_dim);
    m.inv_freq.alloc(half * 4);
    check_cuda(cudaMemcpyAsync(m.inv_freq.p, inv.data(), half * 4, cudaMemcpyHostToDevice, m.stream), "upload");
    check_cuda(cudaStreamSynchronize(m.stream), "upload");
  }

  // Embedding tables, f32 (bf16 in a bf16 model).
  void table(DevBuf& dst, int64_t offset_rows, const std::string& name, int64_t rows, int d) {
    const svl_tensor_view& v = need(name, rows * d);
    if (m.tables_bf16) {
      float* src = stage(v);
      launch_f32_to_bf16(src, dst.as<uint8_t>() + offset_rows * d * 2, rows * d, m.stream);
      check_cuda(cudaStreamSynchronize(m.stream), "convert table");
    } else {
      check_cuda(cudaMemcpyAsync(dst.as<uint8_t>() + offset_rows * d * 4, v.data, rows * d * 4,
                                 cudaMemcpyHostToDevice, m.stream),
                 "upload");
      check_cuda(cudaStreamSynchronize(m.stream), "upload");
    }
  }
};

void validate_cfg(const svl_transformer_config& c) {
  auto bad = [](const std::string& m) { throw Error(SVL_ERR_CONFIG, m); };
  if (c.d_model <= 0 || c.num_layers <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 ||
      c.head_dim <= 0)
    bad("non-positive transformer dimension");
  if (c.num_heads % c.num_kv_heads) bad("num_heads must be a multiple of num_kv_heads");
  if (c.head_dim != 64 && c.head_dim != 128)
    throw Error(SVL_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (c.d_model % 32) throw Error(SVL_ERR_UNSUPPORTED, "d_model must be a multiple of 32");
  if (c.ffn_kind < 0 || c.ffn_kind > 2) bad("unknown feed-forward kind");
  if (c.norm_kind < 0 || c.norm_kind > 1) bad("unknown norm kind");
  if (c.weight_dtype < 0 || c.weight_dtype > 3) bad("unknown weight dtype");
  if (c.kv_dtype < 0 || c.kv_dtype > 1) bad("unknown kv dtype");
  if (c.context < 0) bad("negative context");
  if (c.ffn_hidden <= 0) bad("non-positive ffn_hidden");
  if (!(c.max_period > 0)) bad("max_period must be positive");
}

}  // namespace

// The flow head's modulation products (each ResBlock's adaLN_modulation, then the final
// layer's) read the same conditioning, so they run as one product: their packed rows and
// biases are copied, in that order, into m.mods. Packed rows do not depend on the matrix they
// belong to, and every part has a multiple of 4 rows, so the copy keeps the layout (and each
// row's result) of the separate products. The parts stay loaded for their byte counts.
static void stack_mods(Model& m) {
  std::vector<const Linear*> parts;
  for (const ResBlock& r : m.res) parts.push_back(&r.mod);
  parts.push_back(&m.final_mod);
  Linear& S = m.mods;
  const Linear& f = *parts[0];
  S.k = f.k;
  S.wtype = f.wtype;
  S.row_stride = f.row_stride;
  S.n = 0;
  for (const Linear* L : parts) {
    if (L->k != S.k || L->wtype != S.wtype || L->row_stride != S.row_stride || L->n % 4 || !L->bias.p)
      throw Error(SVL_ERR_CONFIG, "flow head modulation products differ in shape");
    S.n += L->n;
  }
  S.w.alloc(S.row_stride * S.n);
  S.bias.alloc((int64_t)S.n * 4);
  int64_t row = 0;
  for (const Linear* L : parts) {
    check_cuda(cudaMemcpyAsync(S.w.as<uint8_t>() + row * S.row_stride, L->w.p, L->row_stride * L->n,
                               cudaMemcpyDeviceToDevice, m.stream), "stack");
    check_cuda(cudaMemcpyAsync(S.bias.as<float>() + row, L->bias.p, (size_t)L->n * 4, cudaMemcpyDeviceToDevice,
                               m.stream), "stack");
    row += L->n;
  }
  check_cuda(cudaStreamSynchronize(m.stream), "stack");
  if (S.wtype == W_BF16 && !make_gemm_operand(S.tc, S.w.p, S.n, S.k, S.row_stride, 128))
    throw Error(SVL_ERR_CUDA, "flow head modulation: cannot encode its TMA tensor map");
}

Model* create_model(int kind, const svl_transformer_config& cfg, const svl_stt_config* stt,
                    const svl_tts_config* tts, const svl_tensor_view* t, int n, int device,
                    const char* prefix) {
  validate_cfg(cfg);
  int count = 0;
  check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) throw Error(SVL_ERR_CUDA, "no such CUDA device");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  gemv_init_device();
  gemm_init_device();
  attention_init_device();
  attention_ref_init_device();
  Model* m = new Model();
  try {
    m->kind = kind;
    m->device = device;
    m->cfg = cfg;
    check_cuda(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "stream");
    Loader ld{*m, t, n, {}};
    const int d = cfg.d_model;
    if (kind == 0) {
      if (!stt) throw Error(SVL_ERR_CONFIG, "missing STT config");
      m->stt = *stt;
      if (stt->n_q < 0 || stt->card <= 0 || stt->text_card <= 0)
        throw Error(SVL_ERR_CONFIG, "invalid STT config");
      // LanguageModel::new (stt/model.rs:196-233).
      m->tables_bf16 = cfg.weight_dtype == SVL_DT_BF16;
      const int elt = m->tables_bf16 ? 2 : 4;
      m->text_emb.alloc((int64_t)(stt->text_card + 1) * d * elt);
      ld.table(m->text_emb, 0, "text_emb.weight", stt->text_card + 1, d);
      m->audio_emb.alloc((int64_t)std::max(stt->n_q, 1) * (stt->card + 1) * d * elt);
      for (int c = 0; c < stt->n_q; c++)
        ld.table(m->audio_emb, (int64_t)c * (stt->card + 1), "emb." + std::to_string(c) + ".weight",
                 stt->card + 1, d);
      m->weight_bytes += (int64_t)(1 + stt->n_q) * d * elt;  // rows read per step
      ld.transformer("transformer.");
      m->out_norm.kind = NORM_RMS;
      m->out_norm.eps = 1e-8f;
      m->out_norm.w = ld.vec("out_norm.alpha", d);
      ld.linear(m->text_linear, "text_linear.weight", "", stt->text_card, d, true);
      m->extra.resize(std::max(stt->extra_heads_num, 0));
      for (int i = 0; i < stt->extra_heads_num; i++)
        ld.linear(m->extra[i], "extra_heads." + std::to_string(i) + ".weight", "",
                  stt->extra_heads_dim, d, false);
    } else if (kind == 2) {
      // A bare Transformer::new (nn/transformer.rs:106-125) under `prefix`: the transformer
      // of Mimi's ProjectedTransformer (nn/mimi.rs:74-112), no embedding and no head.
      ld.transformer(prefix ? prefix : "transformer.");
    } else {
      // FlowLm::new (tts/flow_lm.rs:45-126), english config: no z_proj, no low-rank table.
      if (!tts) throw Error(SVL_ERR_CONFIG, "missing TTS config");
      m->tts = *tts;
      const int lat = tts->latent_dim, dim = tts->flow_dim;
      if (lat <= 0 || lat % 32 || dim <= 0 || dim % 32 || dim > 1024 || tts->flow_depth < 0 ||
          tts->text_bins <= 0 || tts->flow_kind < 0 || tts->flow_kind > 3)
        throw Error(SVL_ERR_CONFIG, "invalid TTS config");
      m->cond_table = ld.vec("conditioner.embed.weight", (int64_t)(tts->text_bins + 1) * d);
      ld.linear(m->input_linear, "input_linear.weight", "", d, lat, true);
      ld.transformer("transformer.");
      m->out_norm.kind = NORM_LAYER;
      m->out_norm.eps = 1e-5f;
      m->out_norm.w = ld.vec("out_norm.weight", d);
      m->out_norm.b = ld.vec("out_norm.bias", d);
      m->eos_w = ld.vec("out_eos.weight", d);
      m->eos_b = ld.vec("out_eos.bias", 1);
      m->bos = ld.vec("bos_emb", lat);
      // FlowHead::new (tts/flow_lm.rs:239-257).
      const int n_time = tts->flow_kind == 0 ? 2 : tts->flow_kind == 1 ? 1 : 0;
      m->time_emb.resize(n_time);
      for (int i = 0; i < n_time; i++) {
        TimeEmbed& e = m->time_emb[i];
        const std::string p = "flow_net.time_embed." + std::to_string(i) + ".";
        e.freqs = ld.vec(p + "freqs", 128);
        ld.linear(e.l1, p + "mlp.0.weight", p + "mlp.0.bias", dim, 256, false);
        ld.linear(e.l2, p + "mlp.2.weight", p + "mlp.2.bias", dim, dim, false);
        e.alpha = ld.vec(p + "mlp.3.alpha", dim);
      }
      ld.linear(m->cond_embed, "flow_net.cond_embed.weight", "flow_net.cond_embed.bias", dim, d, true);
      ld.linear(m->input_proj, "flow_net.input_proj.weight", "flow_net.input_proj.bias", dim, lat, true);
      m->res.resize(tts->flow_depth);
      for (int i = 0; i < tts->flow_depth; i++) {
        ResBlock& r = m->res[i];
        const std::string p = "flow_net.res_blocks." + std::to_string(i) + ".";
        r.ln.kind = NORM_LAYER;
        r.ln.eps = 1e-6f;
        r.ln.w = ld.vec(p + "in_ln.weight", dim);
        r.ln.b = ld.vec(p + "in_ln.bias", dim);
        ld.linear(r.mlp1, p + "mlp.0.weight", p + "mlp.0.bias", dim, dim, true);
        ld.linear(r.mlp2, p + "mlp.2.weight", p + "mlp.2.bias", dim, dim, true);
        ld.linear(r.mod, p + "adaLN_modulation.1.weight", p + "adaLN_modulation.1.bias", 3 * dim, dim, true);
      }
      ld.linear(m->final_mod, "flow_net.final_layer.adaLN_modulation.1.weight",
                "flow_net.final_layer.adaLN_modulation.1.bias", 2 * dim, dim, true);
      ld.linear(m->final_linear, "flow_net.final_layer.linear.weight",
                "flow_net.final_layer.linear.bias", lat, dim, true);
      stack_mods(*m);
    }
    check_cuda(cudaStreamSynchronize(m->stream), "load");
  } catch (...) {
    delete m;
    throw;
  }
  return m;
}

// Many streams over Q8_0 / Q4_1 weights run on the tensor cores from f16 images of the
// dequantised matrices, built once per model when the first such state is created (the
// packed weights stay in use for small batches). The images hold the values the quantised
// dot products use (q * d, or d * q + m) rounded to f16 (11 significant bits: the products
// of a 7-bit integer and an f16 scale lose at most 2^-12), and cost 2 bytes per weight of
// device memory. The activations meet them as f16 values of their Q8 blocks.
void ensure_shadows(Model& m) {
  std::lock_guard<std::mutex> lock(m.shadow_mu);
  if (m.shadows) return;
  auto shadow = [&](Linear& L) {
    if (L.wtype != W_Q8 && L.wtype != W_Q4) return;
    const int64_t stride = packed_row_stride(W_BF16, L.k);
    L.shadow.alloc(stride * L.n);
    launch_dequant_bf16(L.w.as<uint8_t>(), L.row_stride, L.n, L.k, L.wtype, L.shadow.p, stride, m.stream, 1);
    if (!make_gemm_operand(L.tc, L.shadow.p, L.n, L.k, stride, 128, 1))
      throw Error(SVL_ERR_CUDA, "cannot encode the TMA tensor map of a dequantised matrix");
  };
  for (Layer& L : m.layers) {
    shadow(L.in_proj);
    shadow(L.out_proj);
    shadow(L.ff1);
    shadow(L.ff2);
  }
  if (m.kind == 0) shadow(m.text_linear);
  check_cuda(cudaStreamSynchronize(m.stream), "dequantise");
  m.shadows = true;
}

void queue_error_read(State& s, cudaStream_t st) {
  check_cuda(cudaMemcpyAsync(s.h_err.p, s.err.p, 4, cudaMemcpyDeviceToHost, st), "d2h");
}

void raise_device_error(State& s, cudaStream_t st) {
  const int e = *s.h_err.as<int>();
  if (!e) return;
  *s.h_err.as<int>() = 0;
  check_cuda(cudaMemsetAsync(s.err.p, 0, 4, st), "memset");
  check_cuda(cudaStreamSynchronize(st), "sync");
  if (e == 1) throw Error(SVL_ERR_INVALID_INPUT, "a token id out of range reached the device");
  throw Error(SVL_ERR_TIMEOUT, "a bounded device-side wait ran out (code " + std::to_string(e) + ")");
}

// Positions a reference-order state's RoPE table covers when max_positions does not say.
constexpr int kRefRopePositions = 8192;

State* create_state(Model* m, int max_batch, int max_positions, uint32_t flags) {
  if (max_batch <= 0) throw Error(SVL_ERR_INVALID_INPUT, "max_batch must be positive");
  check_cuda(cudaSetDevice(m->device), "cudaSetDevice");
  const auto& c = m->cfg;
  State* s = new State();
  try {
    s->m = m;
    s->max_batch = max_batch;
    s->windowed = c.context > 0;
    s->cap = s->windowed ? c.context : max_positions;
    if (s->cap <= 0) throw Error(SVL_ERR_INVALID_INPUT, "max_positions must be positive without a window");
    s->ref_order = (flags & SVL_STATE_REFERENCE_ORDER) != 0;
    s->test_withheld_copy = (flags & SVL_STATE_TEST_WITHHELD_COPY) != 0;
    if (s->ref_order) {
      if (!attention_ref_supported(c.head_dim, s->cap))
        throw Error(SVL_ERR_UNSUPPORTED, "reference order: the ring is too long for the in-order attention");
      // (cos, sin)(pos * inv_freq[i]) with the C library's cosf / sinf, as the reference's
      // forward_block evaluates its RoPE table (nn/transformer.rs:159-166).
      const int half = c.head_dim / 2;
      s->rope_positions = std::max(max_positions, kRefRopePositions);
      std::vector<float> inv(half), tab((size_t)s->rope_positions * half * 2);
      check_cuda(cudaMemcpy(inv.data(), m->inv_freq.p, half * 4, cudaMemcpyDeviceToHost), "d2h");
      for (int pos = 0; pos < s->rope_positions; pos++)
        for (int i = 0; i < half; i++) {
          const float f = (float)pos * inv[i];
          tab[((size_t)pos * half + i) * 2] = cosf(f);
          tab[((size_t)pos * half + i) * 2 + 1] = sinf(f);
        }
      s->rope_tab.alloc(tab.size() * 4);
      check_cuda(cudaMemcpyAsync(s->rope_tab.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, m->stream), "upload");
      check_cuda(cudaStreamSynchronize(m->stream), "upload");
    }
    s->kv_elt = c.kv_dtype == SVL_DT_BF16 ? 2 : 4;
    s->ring_stream_stride = (int64_t)c.num_kv_heads * s->cap * c.head_dim;
    s->ring_layer_stride = s->ring_stream_stride * max_batch;
    const int64_t ring_bytes = s->ring_layer_stride * c.num_layers * s->kv_elt;
    s->k_ring.alloc(ring_bytes);
    s->v_ring.alloc(ring_bytes);
    check_cuda(cudaMemsetAsync(s->k_ring.p, 0, ring_bytes, m->stream), "memset");
    check_cuda(cudaMemsetAsync(s->v_ring.p, 0, ring_bytes, m->stream), "memset");
    s->pos.alloc(max_batch * 4);
    check_cuda(cudaMemsetAsync(s->pos.p, 0, max_batch * 4, m->stream), "memset");
    s->hpos.assign(max_batch, 0);
    const int d = c.d_model, qd = c.num_heads * c.head_dim;
    s->x.alloc((int64_t)max_batch * d * 4);
    s->q.alloc((int64_t)max_batch * qd * 4);
    s->attn.alloc((int64_t)max_batch * qd * 4);
    s->act.alloc((int64_t)max_batch * c.ffn_hidden * 4);
    // Split the keys of a (stream, head) over a cluster of CTAs so that small batches still
    // cover the SMs.
    const int units = max_batch * c.num_heads;
    int splits = (148 + units - 1) / units;
    splits = std::max(1, std::min({splits, (s->cap + 15) / 16, attention_max_splits()}));
    s->splits = splits;
    if (splits > 1) {
      // Few streams: when every chunk fits attn_flat_kernel's keys per CTA at about two CTAs
      // per SM (at least 8 keys per chunk), flat chunks replace the clusters.
      int fs = std::max(1, 2 * 148 / units);
      fs = std::min(fs, (s->cap + 7) / 8);
      if (fs > 1 && (s->cap + fs - 1) / fs <= attention_flat_max_keys()) {
        s->attn_flat = true;
        s->splits = fs;
        s->attn_part.alloc((int64_t)units * fs * (c.head_dim + 4) * 4);
        s->attn_ticket.alloc((int64_t)units * 4);
        check_cuda(cudaMemsetAsync(s->attn_ticket.p, 0, s->attn_ticket.bytes, m->stream), "memset");
      }
    }
    if (splits == 1) {
      // Many streams: pieces of keys spread over the warps, partials merged per unit.
      s->piece = attention_piece(c.head_dim, s->kv_elt == 2, s->cap, &s->npieces);
      s->attn_part.alloc((int64_t)units * s->npieces * (c.head_dim + 4) * 4);
      if (s->kv_elt == 2) {
        const int64_t rows = (int64_t)max_batch * c.num_kv_heads * s->cap;
        const int box = attention_chunk_keys(c.head_dim, 1);
        s->ring_maps = rows < (int64_t)1 << 31 &&
                       make_ring_map(s->kmap, s->k_ring.p, rows, c.head_dim, c.num_layers, s->ring_layer_stride, box) &&
                       make_ring_map(s->vmap, s->v_ring.p, rows, c.head_dim, c.num_layers, s->ring_layer_stride, box);
      }
    }
    // Argmax candidates: [stream][CTA] of the matrix-vector head, [stream][row tile] of the
    // tensor-core head.
    int64_t cand = kMaxNbChunk * kLogitsGrid;
    if (m->kind == 0) cand = std::max<int64_t>(cand, (int64_t)max_batch * ((m->stt.text_card + 127) / 128));
    s->am_val.alloc(cand * 4);
    s->am_idx.alloc(cand * 4);
    const bool quantised = c.weight_dtype == SVL_DT_Q8_0 || c.weight_dtype == SVL_DT_Q4_1;
    if ((c.weight_dtype == SVL_DT_BF16 || quantised) && max_batch >= kGemmMinBatch && !s->ref_order) {
      if (quantised) ensure_shadows(*m);
      const int kx = std::max({d, qd, m->kind == 1 ? m->tts.flow_dim : 0, m->kind == 1 ? m->tts.latent_dim : 0});
      s->xa.alloc((int64_t)max_batch * kx * 2);
      s->xh.alloc((int64_t)max_batch * c.ffn_hidden * 2);
      check_cuda(cudaMemsetAsync(s->xa.p, 0, s->xa.bytes, m->stream), "memset");
      check_cuda(cudaMemsetAsync(s->xh.p, 0, s->xh.bytes, m->stream), "memset");
      s->rope_cs.alloc((int64_t)max_batch * (c.head_dim / 2) * 8);
      s->gemm_ws.alloc(gemm_workspace_bytes());
      const int bns[3] = {64, 128, 256};
      for (int i = 0; i < 3; i++) {
        const int f16 = quantised ? 1 : 0;
        bool ok = make_gemm_operand(s->xa_d[i], s->xa.p, max_batch, d, (int64_t)d * 2, bns[i], f16) &&
                  make_gemm_operand(s->xa_q[i], s->xa.p, max_batch, qd, (int64_t)qd * 2, bns[i], f16) &&
                  make_gemm_operand(s->xh_f[i], s->xh.p, max_batch, c.ffn_hidden,
                                    (int64_t)c.ffn_hidden * 2, bns[i], f16);
        if (!ok) throw Error(SVL_ERR_CUDA, "cannot encode the TMA tensor maps of the GEMM operands");
      }
    }
    s->am_ticket.alloc(4);
    check_cuda(cudaMemsetAsync(s->am_ticket.p, 0, 4, m->stream), "memset");
    s->err.alloc(4);
    check_cuda(cudaMemsetAsync(s->err.p, 0, 4, m->stream), "memset");
    s->h_err.alloc(4);
    *s->h_err.as<int>() = 0;

    if (m->kind == 0) {
      const auto& st = m->stt;
      s->logits.alloc((int64_t)max_batch * st.text_card * 4);
      s->tok_in.alloc(max_batch * 4);
      s->tok_out.alloc(max_batch * 4);
      s->audio_in.alloc((int64_t)max_batch * std::max(st.n_q, 1) * 4);
      if (st.extra_heads_num > 0) {
        s->extra_logits.alloc((int64_t)max_batch * st.extra_heads_num * st.extra_heads_dim * 4);
        s->extra_p.alloc((int64_t)max_batch * st.extra_heads_num * 4);
      }
      s->h_tok_in.alloc(max_batch * 4);
      s->h_tok_out.alloc(max_batch * 4);
      s->h_audio_in.alloc((int64_t)max_batch * std::max(st.n_q, 1) * 4);
    }
    if (m->kind == 1) {
      const auto& t = m->tts;
      const int64_t B = max_batch, lat = t.latent_dim, dim = t.flow_dim;
      s->latent_in.alloc(B * lat * 4);
      s->noise.alloc(B * lat * 4);
      s->latent_out.alloc(B * lat * 4);
      s->tmp.alloc(B * lat * 4);
      s->eos.alloc(B * 4);
      s->z.alloc(B * d * 4);
      s->y.alloc(B * dim * 4);
      s->sy.alloc(B * dim * 4);
      s->hbuf.alloc(B * dim * 4);
      s->h2buf.alloc(B * dim * 4);
      s->xs2.alloc(B * dim * 4);
      s->modbuf.alloc(B * m->mods.n * 4);
      s->temb_in.alloc(256 * 4);
      s->temb_h.alloc(dim * 4);
      s->temb_o.alloc(dim * 4);
    }
    // tok_out holds each stream's last argmax (the text token a resumed stream feeds back).
    if (m->kind == 0) check_cuda(cudaMemsetAsync(s->tok_out.p, 0, max_batch * 4, m->stream), "memset");
    check_cuda(cudaStreamSynchronize(m->stream), "state init");
  } catch (...) {
    delete s;
    throw;
  }
  return s;
}

namespace {

GemvParams gemv_base(const Linear& L, const float* x, int64_t x_stride, int nb) {
  GemvParams p{};
  p.w = L.w.as<uint8_t>();
  p.row_stride = L.row_stride;
  p.n = L.n;
  p.k = L.k;
  p.wtype = L.wtype;
  p.x = x;
  p.x_stride = x_stride;
  p.nb = nb;
  p.norm = NORM_NONE;
  p.bias = L.bias.as<float>();
  return p;
}

GemvParams gemv_base(const Linear& L, const float* x, int64_t x_stride, int nb, const State& s) {
  GemvParams p = gemv_base(L, x, x_stride, nb);
  p.ref_order = s.ref_order;
  p.err = s.err.as<int>();
  return p;
}

void set_norm(GemvParams& p, const Norm& N) {
  p.norm = N.kind;
  p.norm_w = N.w.as<float>();
  p.norm_b = N.b.as<float>();
  p.eps = N.eps;
}

// L2 prefetches. A small-batch kernel that reads its data cold from HBM gets ~3.5 TB/s (a burst
// of tens of KB per SM waits ~1.6 us for its first bytes); data prefetched into L2 shortly
// before comes at ~6-7 TB/s, but with plain accesses it is gone again after some 64 MB of
// other traffic (measured on B200 with bulk copies of 96 KB per SM). So every kernel of the
// step pulls into L2 the data of the kernel kPrefetchDistance places after it in the step's
// sequence -- per layer in_proj, attention (the layer's K and V rings), out_proj, linear_in,
// linear_out, then the STT head -- counted cyclically, the next step's first kernels after the
// head. The prefetches carry an evict-last policy and the kernels' own reads of their weights
// and keys an evict-first one, so the reads streaming through L2 in between no longer push the
// prefetched lines out. Measured per STT-1b q8_0 step at batch 1 (full window): without the
// policies 639 us at distance 2; with them 615 us at distance 2, 611 at 3, 616 at 4, 619 at 5.
// A range is prefetched only when it takes at most a quarter of L2.
constexpr int64_t kPrefetchMax = 32ll * 1024 * 1024;
constexpr int kPrefetchDistance = 3;

PrefetchRange weights_range(const Linear* L) {
  if (!L || L->row_stride * L->n > kPrefetchMax) return PrefetchRange{};
  return PrefetchRange{L->w.as<uint8_t>(), L->row_stride * L->n};
}

// Layer l's K (v = 0) or V (v = 1) ring of streams [b0, b0 + nb): one contiguous run.
PrefetchRange ring_range(const State& s, int l, int b0, int nb, int v) {
  const int64_t bytes = (int64_t)nb * s.ring_stream_stride * s.kv_elt;
  if (bytes > kPrefetchMax) return PrefetchRange{};
  const DevBuf& r = v ? s.v_ring : s.k_ring;
  return PrefetchRange{r.as<uint8_t>() + ((int64_t)l * s.ring_layer_stride + (int64_t)b0 * s.ring_stream_stride) * s.kv_elt, bytes};
}

// The prefetches of kernel `idx` of the step (5 per layer: in_proj, attention, out_proj,
// linear_in, linear_out; then the head of an STT model): the data of kernel
// idx + kPrefetchDistance.
void set_prefetch(const Model& m, const State& s, int idx, int b0, int nb, PrefetchRange* pf) {
  const int L = (int)m.layers.size(), n = 5 * L + (m.kind == 0 ? 1 : 0);
  const int t = (idx + kPrefetchDistance) % n;
  for (int i = 0; i < kMaxPrefetch; i++) pf[i] = PrefetchRange{};
  if (t == 5 * L) {
    pf[0] = weights_range(&m.text_linear);
    return;
  }
  const Layer& Lt = m.layers[t / 5];
  switch (t % 5) {
    case 0: pf[0] = weights_range(&Lt.in_proj); break;
    case 1:
      pf[0] = ring_range(s, t / 5, b0, nb, 0);
      pf[1] = ring_range(s, t / 5, b0, nb, 1);
      break;
    case 2: pf[0] = weights_range(&Lt.out_proj); break;
    case 3: pf[0] = weights_range(&Lt.ff1); break;
    default: pf[0] = weights_range(&Lt.ff2); break;
  }
}

}  // namespace

void enqueue_layers_mask(Model& m, State& s, int b0, int nb, cudaStream_t st, bool do_lin,
                         bool do_attn);

bool use_tensor_cores(const Model& m, const State& s, int nb) {
  return (m.cfg.weight_dtype == SVL_DT_BF16 || m.shadows) && nb >= kGemmMinBatch && s.xa.p != nullptr;
}

namespace {
int tile_index(int nb) {
  const int bn = gemm_stream_tile(nb);
  return bn == 64 ? 0 : bn == 128 ? 1 : 2;
}
}  // namespace

void enqueue_layers(Model& m, State& s, int b0, int nb, cudaStream_t st) {
  enqueue_layers_mask(m, s, b0, nb, st, true, true);
}

// The parameter blocks of layer l's kernels for streams [b0, b0 + nb): in_proj + RoPE + KV
// write, attention, out_proj + residual, linear_in + activation, linear_out + residual.
LayerParams layer_params(Model& m, State& s, int l, int b0, int nb) {
  const auto& c = m.cfg;
  const int d = c.d_model, hd = c.head_dim, qd = c.num_heads * hd, kvd = c.num_kv_heads * hd;
  float* x = s.x.as<float>() + (int64_t)b0 * d;
  float* q = s.q.as<float>() + (int64_t)b0 * qd;
  float* attn = s.attn.as<float>() + (int64_t)b0 * qd;
  float* act = s.act.as<float>() + (int64_t)b0 * c.ffn_hidden;
  const int* pos = s.pos.as<int>() + b0;
  const Layer& L = m.layers[l];
  uint8_t* kr = s.k_ring.as<uint8_t>() + ((int64_t)l * s.ring_layer_stride + (int64_t)b0 * s.ring_stream_stride) * s.kv_elt;
  uint8_t* vr = s.v_ring.as<uint8_t>() + ((int64_t)l * s.ring_layer_stride + (int64_t)b0 * s.ring_stream_stride) * s.kv_elt;
  LayerParams lp;
  // norm1 + in_proj + RoPE + KV-ring write (nn/transformer.rs:329-342).
  GemvParams g = gemv_base(L.in_proj, x, d, nb, s);
  set_norm(g, L.norm1);
  g.epi = EPI_QKV_ROPE;
  g.out = q;
  g.out_stride = qd;
  g.inv_freq = m.inv_freq.as<float>();
  g.pos = pos;
  g.q_dim = qd;
  g.kv_dim = kvd;
  g.head_dim = hd;
  g.ring_cap = s.cap;
  g.windowed = s.windowed;
  g.k_ring = kr;
  g.v_ring = vr;
  g.ring_stream_stride = s.ring_stream_stride;
  g.kv_bf16 = s.kv_elt == 2;
  g.rope_by_pos = s.rope_tab.as<float2>();
  g.rope_positions = s.rope_positions;
  if (l == 0 && s.test_withheld_copy) {
    g.test_withhold = 1;
    g.wait_limit = 1u << 12;
  }
  set_prefetch(m, s, 5 * l, b0, nb, g.pf);
  lp.in_proj = g;
  // Sliding-window attention (nn/kernels/attention.rs:81-169).
  AttnParams& a = lp.attn;
  a = AttnParams{};
  a.q = q;
  a.k_ring = kr;
  a.v_ring = vr;
  a.ring_stream_stride = s.ring_stream_stride;
  a.kv_bf16 = s.kv_elt == 2;
  a.pos = pos;
  a.nb = nb;
  a.heads = c.num_heads;
  a.kv_heads = c.num_kv_heads;
  a.head_dim = hd;
  a.ring_cap = s.cap;
  a.window = c.context;
  a.scale = std::pow((float)hd, -0.5f);
  a.splits = s.splits;
  a.piece = s.piece;
  a.npieces = s.npieces;
  a.part = s.attn_part.as<float>();
  if (s.attn_flat) {
    a.part += (int64_t)b0 * c.num_heads * s.splits * (hd + 4);
    a.ticket = s.attn_ticket.as<unsigned>() + (int64_t)b0 * c.num_heads;
  }
  a.kmap = s.ring_maps ? s.kmap : nullptr;
  a.vmap = s.ring_maps ? s.vmap : nullptr;
  a.layer = l;
  a.ring_row0 = b0 * c.num_kv_heads * s.cap;
  a.out = attn;
  a.err = s.err.as<int>();
  set_prefetch(m, s, 5 * l + 1, b0, nb, a.pf);
  // out_proj + residual (nn/transformer.rs:344, :239-243).
  g = gemv_base(L.out_proj, attn, qd, nb, s);
  g.epi = EPI_RESIDUAL;
  g.out = x;
  g.out_stride = d;
  g.ls = L.ls1.as<float>();
  set_prefetch(m, s, 5 * l + 2, b0, nb, g.pf);
  lp.out_proj = g;
  // norm2 + feed-forward (nn/transformer.rs:438-464).
  g = gemv_base(L.ff1, x, d, nb, s);
  set_norm(g, L.norm2);
  g.out = act;
  g.out_stride = c.ffn_hidden;
  g.epi = c.ffn_kind == SVL_FFN_GATED_SILU ? EPI_SWIGLU
          : c.ffn_kind == SVL_FFN_PLAIN_GELU_ERF ? EPI_GELU_ERF : EPI_GELU_TANH;
  set_prefetch(m, s, 5 * l + 3, b0, nb, g.pf);
  lp.ff1 = g;
  g = gemv_base(L.ff2, act, c.ffn_hidden, nb, s);
  g.epi = EPI_RESIDUAL;
  g.out = x;
  g.out_stride = d;
  g.ls = L.ls2.as<float>();
  set_prefetch(m, s, 5 * l + 4, b0, nb, g.pf);
  lp.ff2 = g;
  return lp;
}

void enqueue_layers_mask(Model& m, State& s, int b0, int nb, cudaStream_t st, bool do_lin,
                         bool do_attn) {
  const auto& c = m.cfg;
  const int d = c.d_model, hd = c.head_dim, qd = c.num_heads * hd;
  float* x = s.x.as<float>() + (int64_t)b0 * d;
  const int* pos = s.pos.as<int>() + b0;
  const bool tc = use_tensor_cores(m, s, nb);
  const int ti = tc ? tile_index(nb) : 0;
  const int quant = m.shadows ? 1 : 0;  // the Q8 activation blocks of a quantised model
  float2* rope_cs = tc ? s.rope_cs.as<float2>() + (int64_t)b0 * (hd / 2) : nullptr;
  if (tc && do_lin) launch_rope_table(pos, nb, m.inv_freq.as<float>(), hd / 2, rope_cs, st);
  for (int l = 0; l < c.num_layers; l++) {
    const Layer& L = m.layers[l];
    LayerParams lp = layer_params(m, s, l, b0, nb);
    GemvParams g = lp.in_proj;
    g.rope_cs = rope_cs;
    if (do_lin && tc) {
      launch_prep_bf16(x, d, nb, L.norm1.kind, L.norm1.w.as<float>(), L.norm1.b.as<float>(),
                       L.norm1.eps, d, s.xa.p, d, st, quant, quant);
      launch_gemm(g, L.in_proj.tc, s.xa_d[ti], 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
    } else if (do_lin) {
      launch_gemv(g, st);
    }
    if (do_attn) {
      if (s.ref_order)
        launch_attention_ref(lp.attn, st);
      else
        launch_attention_decode(lp.attn, st);
    }
    if (!do_lin) continue;
    g = lp.out_proj;
    if (tc) {
      launch_prep_bf16(lp.attn.out, qd, nb, NORM_NONE, nullptr, nullptr, 0.f, qd, s.xa.p, qd, st, quant, quant);
      launch_gemm(g, L.out_proj.tc, s.xa_q[ti], 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
    } else {
      launch_gemv(g, st);
    }
    g = lp.ff1;
    if (tc) {
      launch_prep_bf16(x, d, nb, L.norm2.kind, L.norm2.w.as<float>(), L.norm2.b.as<float>(),
                       L.norm2.eps, d, s.xa.p, d, st, quant, quant);
      if (quant) {
        // f32 hidden rows, then their Q8 activation blocks as the operand of linear_out.
        launch_gemm(g, L.ff1.tc, s.xa_d[ti], 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
        launch_prep_bf16(g.out, c.ffn_hidden, nb, NORM_NONE, nullptr, nullptr, 0.f, c.ffn_hidden,
                         s.xh.p, c.ffn_hidden, st, 1, 1);
      } else {
        g.out = s.xh.as<float>();  // bf16 hidden rows, the operand of linear_out
        launch_gemm(g, L.ff1.tc, s.xa_d[ti], 0, 1, s.err.as<int>(), s.gemm_ws.as<float>(), st);
      }
    } else {
      launch_gemv(g, st);
    }
    g = lp.ff2;
    if (tc)
      launch_gemm(g, L.ff2.tc, s.xh_f[ti], 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
    else
      launch_gemv(g, st);
  }
}

void launch_extra_heads(const float* logits, int nb, int heads, int dim, float* out,
                        cudaStream_t st);

namespace {

GemvParams head_params(Model& m, State& s, int nb) {
  GemvParams g = gemv_base(m.text_linear, s.x.as<float>(), m.cfg.d_model, nb, s);
  set_norm(g, m.out_norm);
  g.epi = EPI_LOGITS;
  g.out = s.logits.as<float>();
  g.out_stride = m.stt.text_card;
  g.am_val = s.am_val.as<float>();
  g.am_idx = s.am_idx.as<int>();
  g.am_ticket = s.am_ticket.as<unsigned>();
  g.tokens = s.tok_out.as<uint32_t>();
  set_prefetch(m, s, 5 * (int)m.layers.size(), 0, nb, g.pf);
  return g;
}

}  // namespace

// The logits product with its argmax: on the tensor cores (out_norm as the operand prep)
// when the step's products run there.
void launch_head(Model& m, State& s, const GemvParams& g, cudaStream_t st) {
  if (use_tensor_cores(m, s, g.nb)) {
    const int d = m.cfg.d_model;
    launch_prep_bf16(g.x, d, g.nb, m.out_norm.kind, m.out_norm.w.as<float>(),
                     m.out_norm.b.as<float>(), m.out_norm.eps, d, s.xa.p, d, st,
                     m.shadows ? 1 : 0, m.shadows ? 1 : 0);
    launch_gemm(g, m.text_linear.tc, s.xa_d[tile_index(g.nb)], 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
  } else {
    launch_gemv(g, st);
  }
}

void enqueue_stt_step(Model& m, State& s, int nb, cudaStream_t st) {
  const auto& c = m.cfg;
  const int d = c.d_model;
  EmbedParams e{};
  e.text_table = m.text_emb.p;
  e.audio_tables = m.audio_emb.p;
  e.tables_bf16 = m.tables_bf16;
  e.text_tok = s.tok_in.as<uint32_t>();
  e.audio_tok = s.audio_in.as<uint32_t>();
  e.nb = nb;
  e.d = d;
  e.n_q = m.stt.n_q;
  e.card = m.stt.card;
  e.text_card = m.stt.text_card;
  e.x = s.x.as<float>();
  e.error_flag = s.err.as<int>();
  launch_embed(e, st);
  enqueue_layers(m, s, 0, nb, st);
  // out_norm + text_linear + argmax (stt/model.rs:252-258). The step's last reader of the
  // positions is done once the argmax is final: the argmax's last CTA advances them.
  GemvParams g = head_params(m, s, nb);
  g.pos_advance = s.pos.as<int>();
  launch_head(m, s, g, st);
  // Extra (VAD) heads: softmax p[0] of each (stt/model.rs:259-271); never quantised.
  const int eh = m.stt.extra_heads_num, edim = m.stt.extra_heads_dim;
  for (int i = 0; i < eh; i++) {
    GemvParams h = gemv_base(m.extra[i], s.x.as<float>(), d, nb, s);
    set_norm(h, m.out_norm);
    h.epi = EPI_STORE;
    h.out = s.extra_logits.as<float>() + i * edim;
    h.out_stride = (int64_t)eh * edim;
    launch_gemv(h, st);
  }
  if (eh > 0) launch_extra_heads(s.extra_logits.as<float>(), nb, eh, edim, s.extra_p.as<float>(), st);
}

namespace {

// Captures fn's launches on st into a graph stored under key (if not captured yet); returns
// the graph's kernel nodes (the launches one replay makes).
template <class F>
int capture_graph(State& s, int key, cudaStream_t st, F&& fn) {
  auto it = s.graphs.find(key);
  if (it != s.graphs.end()) return s.graph_kernels[key];
  cudaGraph_t graph = nullptr;
  check_cuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    fn();
  } catch (...) {
    cudaStreamEndCapture(st, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  check_cuda(cudaStreamEndCapture(st, &graph), "end capture");
  size_t n = 0;
  int kernels = 0;
  cudaError_t e = cudaGraphGetNodes(graph, nullptr, &n);
  if (e == cudaSuccess && n) {
    std::vector<cudaGraphNode_t> nodes(n);
    e = cudaGraphGetNodes(graph, nodes.data(), &n);
    for (size_t i = 0; e == cudaSuccess && i < n; i++) {
      cudaGraphNodeType t;
      e = cudaGraphNodeGetType(nodes[i], &t);
      if (e == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
    }
  }
  cudaGraphExec_t exec = nullptr;
  if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  check_cuda(e, "graph instantiate");
  s.graphs.emplace(key, exec);
  s.graph_kernels[key] = kernels;
  return kernels;
}

}  // namespace

int capture_stt_graph(Model& m, State& s, int nb, cudaStream_t st) {
  return capture_graph(s, nb, st, [&] { enqueue_stt_step(m, s, nb, st); });
}

void launch_stt_graph(Model& m, State& s, int nb, cudaStream_t st) {
  capture_stt_graph(m, s, nb, st);
  check_cuda(cudaGraphLaunch(s.graphs[nb], st), "graph launch");
}

// ---- Pocket-TTS step ------------------------------------------------------------------

namespace {

// bf16 operand map over the state's xa buffer for rows of k elements, tiles of bn streams.
const GemmOperand& xa_map(State& s, int k, int nb) {
  const int bn = gemm_stream_tile(nb);
  const int64_t key = (int64_t)k * 512 + bn;
  auto it = s.xa_by_k.find(key);
  if (it == s.xa_by_k.end()) {
    GemmOperand op;
    if (!make_gemm_operand(op, s.xa.p, s.max_batch, k, (int64_t)k * 2, bn))
      throw Error(SVL_ERR_CUDA, "cannot encode a TMA tensor map of a GEMM operand");
    it = s.xa_by_k.emplace(key, op).first;
  }
  return it->second;
}

// One weight product over streams [0, nb): out[b] = epi(L . x[b] + bias). The matrix-vector
// kernel reads the f32 rows directly; for many bf16 streams the rows become bf16 operand rows
// and the product runs on the tensor cores.
void linear_fwd(Model& m, State& s, const Linear& L, const float* x, int64_t x_stride, int nb,
                int epi, float* out, int64_t out_stride, cudaStream_t st) {
  GemvParams g = gemv_base(L, x, x_stride, nb, s);
  g.epi = epi;
  g.out = out;
  g.out_stride = out_stride;
  if (use_tensor_cores(m, s, nb) && L.tc.valid) {
    launch_prep_bf16(x, x_stride, nb, NORM_NONE, nullptr, nullptr, 0.f, L.k, s.xa.p, L.k, st);
    launch_gemm(g, L.tc, xa_map(s, L.k, nb), 0, 0, s.err.as<int>(), s.gemm_ws.as<float>(), st);
  } else {
    launch_gemv(g, st);
  }
}

// FlowHead::forward (tts/flow_lm.rs:259-287) and decode (:290-315) from s.z into the latent
// s.latent_out (which enters holding the noise).
// The flow head's conditioning time input for each decode step i of `steps`: the sum over the
// TimestepEmbedders of their outputs at t = (i + e) / steps (flow_lm.rs:266-275). It is the same
// for every stream and frame, so it is computed once per step count, on st, outside any graph
// capture; null for a head without time embedders.
const float* time_table(Model& m, State& s, int steps, cudaStream_t st) {
  const int n_time = (int)m.time_emb.size();
  if (n_time == 0) return nullptr;
  auto it = s.time_tables.find(steps);
  if (it != s.time_tables.end()) return it->second.as<float>();
  const int dim = m.tts.flow_dim;
  DevBuf tab;
  tab.alloc((int64_t)steps * dim * 4);
  for (int i = 0; i < steps; i++) {
    for (int e = 0; e < n_time; e++) {
      const TimeEmbed& te = m.time_emb[e];
      const float tv = (float)(i + e) / (float)steps;
      launch_time_input(te.freqs.as<float>(), tv, s.temb_in.as<float>(), st);
      GemvParams g = gemv_base(te.l1, s.temb_in.as<float>(), 256, 1, s);
      g.epi = EPI_SILU;
      g.out = s.temb_h.as<float>();
      g.out_stride = dim;
      launch_gemv(g, st);
      g = gemv_base(te.l2, s.temb_h.as<float>(), dim, 1, s);
      g.epi = EPI_STORE;
      g.out = s.temb_o.as<float>();
      g.out_stride = dim;
      launch_gemv(g, st);
      launch_time_norm(s.temb_o.as<float>(), dim, te.alpha.as<float>(), tab.as<float>() + (int64_t)i * dim,
                       e == 0, st);
    }
  }
  check_cuda(cudaGetLastError(), "time table");
  check_cuda(cudaStreamSynchronize(st), "time table");  // complete before any other stream reads it
  return s.time_tables.emplace(steps, std::move(tab)).first->second.as<float>();
}

void enqueue_flow(Model& m, State& s, int nb, int steps, const float* ttab, cudaStream_t st) {
  const auto& t = m.tts;
  const int dim = t.flow_dim, lat = t.latent_dim, d = m.cfg.d_model;
  const int n_time = (int)m.time_emb.size();
  float* y = s.y.as<float>();
  float* sy = s.sy.as<float>();
  float* xs = s.xs2.as<float>();
  float* hh = s.hbuf.as<float>();
  float* h2 = s.h2buf.as<float>();
  float* mod = s.modbuf.as<float>();
  float* x = s.latent_out.as<float>();
  float* flow = s.tmp.as<float>();
  // cond_embed does not depend on the decode step.
  linear_fwd(m, s, m.cond_embed, s.z.as<float>(), d, nb, EPI_STORE, y, dim, st);
  const int iters = n_time > 0 ? steps : 1;
  for (int i = 0; i < iters; i++) {
    // TimestepEmbedder per time (lsd: i/steps and (i+1)/steps; flow matching: i/steps),
    // summed: row i of the step count's time table.
    launch_cond_silu(y, n_time > 0 ? ttab + (int64_t)i * dim : nullptr,
                     n_time > 0 ? (float)(1.0 / (double)n_time) : 0.f, dim, nb, sy, st);
    linear_fwd(m, s, m.input_proj, x, lat, nb, EPI_STORE, xs, dim, st);
    // Every block's shift / scale / gate and the final layer's shift / scale in one product.
    const int ms = m.mods.n;
    linear_fwd(m, s, m.mods, sy, dim, nb, EPI_STORE, mod, ms, st);
    for (size_t i = 0; i < m.res.size(); i++) {
      const ResBlock& r = m.res[i];
      const float* mi = mod + (int64_t)i * 3 * dim;
      launch_adaln(xs, nb, dim, r.ln.w.as<float>(), r.ln.b.as<float>(), 1, r.ln.eps, mi, ms, hh, st);
      linear_fwd(m, s, r.mlp1, hh, dim, nb, EPI_SILU, h2, dim, st);
      linear_fwd(m, s, r.mlp2, h2, dim, nb, EPI_STORE, hh, dim, st);
      launch_gate_add(xs, mi, ms, 2 * dim, hh, nb, dim, st);
    }
    launch_adaln(xs, nb, dim, nullptr, nullptr, 0, 1e-6f, mod + (int64_t)m.res.size() * 3 * dim, ms, hh, st);
    linear_fwd(m, s, m.final_linear, hh, dim, nb, EPI_STORE, flow, lat, st);
    const int mode = n_time > 0 ? 0 : t.flow_kind == 2 ? 1 : 2;
    launch_flow_update(x, flow, (int64_t)nb * lat, mode, (float)(1.0 / (double)steps), st);
  }
}

// FlowLm::step (tts/flow_lm.rs:162-185) for streams [0, nb).
void enqueue_tts_step(Model& m, State& s, int nb, int steps, const float* ttab, cudaStream_t st) {
  const int d = m.cfg.d_model, lat = m.tts.latent_dim;
  linear_fwd(m, s, m.input_linear, s.latent_in.as<float>(), lat, nb, EPI_STORE, s.x.as<float>(), d, st);
  enqueue_layers(m, s, 0, nb, st);
  launch_advance_positions(s.pos.as<int>(), nb, st);
  launch_tts_head(s.x.as<float>(), nb, d, m.out_norm.w.as<float>(), m.out_norm.b.as<float>(),
                  m.out_norm.eps, m.eos_w.as<float>(), m.eos_b.as<float>(), s.z.as<float>(),
                  s.eos.as<float>(), st);
  check_cuda(cudaMemcpyAsync(s.latent_out.p, s.noise.p, (size_t)nb * lat * 4,
                             cudaMemcpyDeviceToDevice, st), "noise");
  enqueue_flow(m, s, nb, steps, ttab, st);
}

}  // namespace

int capture_tts_graph(Model& m, State& s, int nb, int steps, cudaStream_t st) {
  const float* ttab = time_table(m, s, steps, st);  // outside the capture
  return capture_graph(s, nb + (steps << 16), st, [&] { enqueue_tts_step(m, s, nb, steps, ttab, st); });
}

void launch_tts_graph(Model& m, State& s, int nb, int steps, cudaStream_t st) {
  capture_tts_graph(m, s, nb, steps, st);
  check_cuda(cudaGraphLaunch(s.graphs[nb + (steps << 16)], st), "graph launch");
}

void enqueue_tts_prompt(Model& m, State& s, int b0, int nb, const uint32_t* d_tokens, int n,
                        cudaStream_t st) {
  const int d = m.cfg.d_model;
  for (int t = 0; t < n; t++) {
    launch_prompt_embed(m.cond_table.as<float>(), d_tokens, nb, n, t, d, m.tts.text_bins,
                        s.x.as<float>() + (int64_t)b0 * d, s.err.as<int>(), st);
    enqueue_layers(m, s, b0, nb, st);
    launch_advance_positions(s.pos.as<int>() + b0, nb, st);
  }
}

int64_t enqueue_profile(Model& m, State& s, int nb, int which, cudaStream_t st) {
  const auto& c = m.cfg;
  if (which == 0) {
    enqueue_layers_mask(m, s, 0, nb, st, true, false);
    int64_t bytes = 0;
    for (const Layer& L : m.layers)
      bytes += L.in_proj.bytes() + L.out_proj.bytes() + L.ff1.bytes() + L.ff2.bytes();
    if (m.kind == 0) {
      launch_head(m, s, head_params(m, s, nb), st);
      bytes += m.text_linear.bytes();
    }
    return bytes;
  }
  if (which == 2) {
    enqueue_flow(m, s, nb, 1, time_table(m, s, 1, st), st);
    int64_t bytes = m.cond_embed.bytes() + m.input_proj.bytes() + m.final_mod.bytes() + m.final_linear.bytes();
    for (const ResBlock& r : m.res) bytes += r.mod.bytes() + r.mlp1.bytes() + r.mlp2.bytes();
    for (const TimeEmbed& e : m.time_emb) bytes += e.l1.bytes() + e.l2.bytes();
    return bytes;
  }
  enqueue_layers_mask(m, s, 0, nb, st, false, true);
  int64_t bytes = 0;
  for (int b = 0; b < nb; b++) {
    const int fill = c.context > 0 ? std::min(s.hpos[b] + 1, c.context) : s.hpos[b] + 1;
    bytes += (int64_t)c.num_layers * 2 * fill * c.num_kv_heads * c.head_dim * s.kv_elt;
  }
  return bytes;
}

void state_reset(State& s, int stream) {
  const int b0 = stream < 0 ? 0 : stream, b1 = stream < 0 ? s.max_batch : stream + 1;
  // State operations wait for every stream (a step may be in flight on a caller's stream),
  // then transfer in order on the model's stream.
  check_cuda(cudaDeviceSynchronize(), "reset");
  for (int b = b0; b < b1; b++) s.hpos[b] = 0;
  check_cuda(cudaMemcpyAsync(s.pos.as<int>() + b0, s.hpos.data() + b0, (b1 - b0) * 4,
                             cudaMemcpyHostToDevice, s.m->stream),
             "reset");
  check_cuda(cudaStreamSynchronize(s.m->stream), "reset");
}

void state_export(State& s, int stream, int layer, float* k, float* v, int* len) {
  const auto& c = s.m->cfg;
  const int pos = s.hpos[stream];
  const int n = s.windowed ? std::min(pos, s.cap) : pos;
  const int64_t elems = s.ring_stream_stride;
  std::vector<uint8_t> hk(elems * s.kv_elt), hv(elems * s.kv_elt);
  const int64_t off = ((int64_t)layer * s.ring_layer_stride + (int64_t)stream * s.ring_stream_stride) * s.kv_elt;
  check_cuda(cudaDeviceSynchronize(), "export");
  check_cuda(cudaMemcpyAsync(hk.data(), s.k_ring.as<uint8_t>() + off, hk.size(), cudaMemcpyDeviceToHost, s.m->stream), "export");
  check_cuda(cudaMemcpyAsync(hv.data(), s.v_ring.as<uint8_t>() + off, hv.size(), cudaMemcpyDeviceToHost, s.m->stream), "export");
  check_cuda(cudaStreamSynchronize(s.m->stream), "export");
  auto get = [&](const std::vector<uint8_t>& src, int64_t i) -> float {
    if (s.kv_elt == 4) {
      float f;
      std::memcpy(&f, src.data() + i * 4, 4);
      return f;
    }
    uint16_t h;
    std::memcpy(&h, src.data() + i * 2, 2);
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  };
  const int hd = c.head_dim;
  for (int h = 0; h < c.num_kv_heads; h++)
    for (int j = 0; j < n; j++) {
      const int p = pos - n + j;
      const int slot = s.windowed ? p % s.cap : p;
      for (int i = 0; i < hd; i++) {
        const int64_t src = ((int64_t)h * s.cap + slot) * hd + i;
        const int64_t dst = ((int64_t)h * n + j) * hd + i;
        k[dst] = get(hk, src);
        v[dst] = get(hv, src);
      }
    }
  *len = n;
}

void state_import(State& s, int stream, int layer, const float* k, const float* v, int len,
                  int position) {
  const auto& c = s.m->cfg;
  if (len < 0 || position < len) throw Error(SVL_ERR_INVALID_INPUT, "import: need 0 <= len <= position");
  if (!s.windowed && position > s.cap)
    throw Error(SVL_ERR_INVALID_INPUT, "import: position exceeds the state's max_positions");
  check_cuda(cudaDeviceSynchronize(), "import");
  if (len == 0) {
    // Only the position moves; the ring keeps its contents.
    s.hpos[stream] = position;
    check_cuda(cudaMemcpyAsync(s.pos.as<int>() + stream, &position, 4, cudaMemcpyHostToDevice, s.m->stream), "import");
    check_cuda(cudaStreamSynchronize(s.m->stream), "import");
    return;
  }
  const int keep = s.windowed ? std::min(len, s.cap) : len;
  const int hd = c.head_dim;
  const int64_t elems = s.ring_stream_stride;
  std::vector<uint8_t> hk(elems * s.kv_elt, 0), hv(elems * s.kv_elt, 0);
  auto put = [&](std::vector<uint8_t>& dst, int64_t i, float f) {
    if (s.kv_elt == 4) {
      std::memcpy(dst.data() + i * 4, &f, 4);
    } else {
      uint32_t u;
      std::memcpy(&u, &f, 4);
      u += 0x7fffu + ((u >> 16) & 1u);
      uint16_t h = (uint16_t)(u >> 16);
      std::memcpy(dst.data() + i * 2, &h, 2);
    }
  };
  for (int h = 0; h < c.num_kv_heads; h++)
    for (int j = len - keep; j < len; j++) {
      const int p = position - len + j;
      const int slot = s.windowed ? p % s.cap : p;
      for (int i = 0; i < hd; i++) {
        const int64_t src = ((int64_t)h * len + j) * hd + i;
        const int64_t dst = ((int64_t)h * s.cap + slot) * hd + i;
        put(hk, dst, k[src]);
        put(hv, dst, v[src]);
      }
    }
  const int64_t off = ((int64_t)layer * s.ring_layer_stride + (int64_t)stream * s.ring_stream_stride) * s.kv_elt;
  check_cuda(cudaMemcpyAsync(s.k_ring.as<uint8_t>() + off, hk.data(), hk.size(), cudaMemcpyHostToDevice, s.m->stream), "import");
  check_cuda(cudaMemcpyAsync(s.v_ring.as<uint8_t>() + off, hv.data(), hv.size(), cudaMemcpyHostToDevice, s.m->stream), "import");
  s.hpos[stream] = position;
  check_cuda(cudaMemcpyAsync(s.pos.as<int>() + stream, &position, 4, cudaMemcpyHostToDevice, s.m->stream), "import");
  check_cuda(cudaStreamSynchronize(s.m->stream), "import");
}

}  // namespace svl
