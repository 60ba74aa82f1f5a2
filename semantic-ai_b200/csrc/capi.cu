// capi.cu — the extern "C" entry points declared in include/svl_cuda.h.
#include <cstring>
#include <string>
#include <vector>

#include "engine.h"

using svl::Error;

namespace {

thread_local std::string g_err;

svl_status fail(svl_status c, const std::string& msg) {
  g_err = msg;
  return c;
}

template <class F>
svl_status guarded(F&& f) {
  try {
    f();
    return SVL_OK;
  } catch (const Error& e) {
    return fail(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return fail(SVL_ERR_OOM, "host allocation failed");
  } catch (const std::exception& e) {
    return fail(SVL_ERR_CUDA, e.what());
  }
}

void need(bool ok, svl_status c, const char* msg) {
  if (!ok) throw Error(c, msg);
}

void check_stream(svl::State& s, int stream) {
  need(stream >= 0 && stream < s.max_batch, SVL_ERR_INVALID_INPUT, "stream index out of range");
}

// Positions beyond the ring are an error without a window (the reference's cache grows), and
// in reference order positions past the state's RoPE table are not supported.
void check_room(svl::State& s, int b0, int nb, int steps) {
  for (int b = b0; b < b0 + nb; b++) {
    if (!s.windowed && s.hpos[b] + steps > s.cap)
      throw Error(SVL_ERR_INVALID_INPUT, "stream would exceed the state's max_positions");
    if (s.ref_order && s.hpos[b] + steps > s.rope_positions)
      throw Error(SVL_ERR_UNSUPPORTED, "reference order covers positions below " +
                                           std::to_string(s.rope_positions) + " (its RoPE table)");
  }
}
void check_room(svl::State& s, int nb, int steps) { check_room(s, 0, nb, steps); }

}  // namespace

void svl::set_last_error(const std::string& msg) { g_err = msg; }

extern "C" {

SVL_API const char* svl_last_error(void) { return g_err.c_str(); }
SVL_API const char* svl_version(void) { return "svl-b200 0.1 (sm_100a)"; }

SVL_API svl_status svl_stt_model_create(const svl_transformer_config* cfg,
                                        const svl_stt_config* stt,
                                        const svl_tensor_view* tensors, int32_t n_tensors,
                                        int32_t device, svl_model** out) {
  return guarded([&] {
    need(cfg && stt && out && (tensors || n_tensors == 0), SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::Model* m = svl::create_model(0, *cfg, stt, nullptr, tensors, n_tensors, device);
    *out = new svl_model{m};
  });
}

SVL_API svl_status svl_tts_model_create(const svl_transformer_config* cfg,
                                        const svl_tts_config* tts,
                                        const svl_tensor_view* tensors, int32_t n_tensors,
                                        int32_t device, svl_model** out) {
  return guarded([&] {
    need(cfg && tts && out && (tensors || n_tensors == 0), SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::Model* m = svl::create_model(1, *cfg, nullptr, tts, tensors, n_tensors, device);
    *out = new svl_model{m};
  });
}

SVL_API void svl_model_destroy(svl_model* model) {
  if (!model) return;
  cudaSetDevice(model->m->device);
  delete model->m;
  delete model;
}

SVL_API int64_t svl_model_weight_bytes(const svl_model* model) {
  return model ? model->m->weight_bytes : 0;
}

SVL_API svl_status svl_state_create(svl_model* model, int32_t max_batch, int32_t max_positions,
                                    svl_state** out) {
  return guarded([&] {
    need(model && out, SVL_ERR_INVALID_INPUT, "null argument");
    *out = nullptr;
    svl::State* s = svl::create_state(model->m, max_batch, max_positions);
    *out = new svl_state{s, model};
  });
}

SVL_API svl_status svl_state_create_ex(svl_model* model, int32_t max_batch, int32_t max_positions,
                                       uint32_t flags, svl_state** out) {
  return guarded([&] {
    need(model && out, SVL_ERR_INVALID_INPUT, "null argument");
    need((flags & ~(SVL_STATE_REFERENCE_ORDER | SVL_STATE_TEST_WITHHELD_COPY)) == 0, SVL_ERR_INVALID_INPUT,
         "unknown state flags");
    *out = nullptr;
    svl::State* s = svl::create_state(model->m, max_batch, max_positions, flags);
    *out = new svl_state{s, model};
  });
}

SVL_API void svl_state_destroy(svl_state* state) {
  if (!state) return;
  cudaSetDevice(state->s->m->device);
  delete state->s;
  delete state;
}

SVL_API svl_status svl_state_reset(svl_state* state, int32_t stream) {
  return guarded([&] {
    need(state, SVL_ERR_INVALID_INPUT, "null state");
    if (stream >= 0) check_stream(*state->s, stream);
    svl::check_cuda(cudaSetDevice(state->s->m->device), "cudaSetDevice");
    svl::state_reset(*state->s, stream);
  });
}

SVL_API svl_status svl_state_position(svl_state* state, int32_t stream, int32_t* position) {
  return guarded([&] {
    need(state && position, SVL_ERR_INVALID_INPUT, "null argument");
    check_stream(*state->s, stream);
    *position = state->s->hpos[stream];
  });
}

SVL_API svl_status svl_state_copy(svl_state* to, int32_t dst, const svl_state* from, int32_t src) {
  return guarded([&] {
    need(to && from, SVL_ERR_INVALID_INPUT, "null state");
    svl::State& a = *to->s;
    const svl::State& b = *from->s;
    need(a.m == b.m, SVL_ERR_INVALID_INPUT, "states of different models");
    need(a.cap == b.cap, SVL_ERR_INVALID_INPUT, "states of different capacity");
    check_stream(a, dst);
    need(src >= 0 && src < b.max_batch, SVL_ERR_INVALID_INPUT, "stream index out of range");
    svl::check_cuda(cudaSetDevice(a.m->device), "cudaSetDevice");
    svl::check_cuda(cudaDeviceSynchronize(), "copy");
    cudaStream_t st = a.m->stream;
    const int64_t bytes = a.ring_stream_stride * a.kv_elt;
    for (int l = 0; l < a.m->cfg.num_layers; l++) {
      const int64_t da = ((int64_t)l * a.ring_layer_stride + (int64_t)dst * a.ring_stream_stride) * a.kv_elt;
      const int64_t db = ((int64_t)l * b.ring_layer_stride + (int64_t)src * b.ring_stream_stride) * b.kv_elt;
      svl::check_cuda(cudaMemcpyAsync(a.k_ring.as<uint8_t>() + da, b.k_ring.as<uint8_t>() + db, bytes, cudaMemcpyDeviceToDevice, st), "copy");
      svl::check_cuda(cudaMemcpyAsync(a.v_ring.as<uint8_t>() + da, b.v_ring.as<uint8_t>() + db, bytes, cudaMemcpyDeviceToDevice, st), "copy");
    }
    // The stream's last argmax travels with it (the text token a resumed stream feeds back).
    if (a.tok_out.p && b.tok_out.p)
      svl::check_cuda(cudaMemcpyAsync(a.tok_out.as<uint32_t>() + dst, b.tok_out.as<uint32_t>() + src, 4, cudaMemcpyDeviceToDevice, st), "copy");
    a.hpos[dst] = b.hpos[src];
    svl::check_cuda(cudaMemcpyAsync(a.pos.as<int>() + dst, &a.hpos[dst], 4, cudaMemcpyHostToDevice, st), "copy");
    svl::check_cuda(cudaStreamSynchronize(st), "copy");
  });
}

SVL_API svl_status svl_state_export(svl_state* state, int32_t stream, int32_t layer, float* k,
                                    float* v, int32_t* len, int32_t* position) {
  return guarded([&] {
    need(state && k && v && len, SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    check_stream(s, stream);
    need(layer >= 0 && layer < s.m->cfg.num_layers, SVL_ERR_INVALID_INPUT, "layer out of range");
    svl::check_cuda(cudaSetDevice(s.m->device), "cudaSetDevice");
    int n = 0;
    svl::state_export(s, stream, layer, k, v, &n);
    *len = n;
    if (position) *position = s.hpos[stream];
  });
}

SVL_API svl_status svl_state_import(svl_state* state, int32_t stream, int32_t layer,
                                    const float* k, const float* v, int32_t len,
                                    int32_t position) {
  return guarded([&] {
    need(state && (len == 0 || (k && v)), SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    check_stream(s, stream);
    need(layer >= 0 && layer < s.m->cfg.num_layers, SVL_ERR_INVALID_INPUT, "layer out of range");
    svl::check_cuda(cudaSetDevice(s.m->device), "cudaSetDevice");
    svl::state_import(s, stream, layer, k, v, len, position);
  });
}

SVL_API svl_status svl_voice_save(svl_state* state, int32_t stream, const char* path) {
  return guarded([&] {
    need(state && path, SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    check_stream(s, stream);
    svl::check_cuda(cudaSetDevice(s.m->device), "cudaSetDevice");
    svl::voice_save(s, stream, path);
  });
}

SVL_API svl_status svl_voice_load(svl_state* state, const int32_t* streams, int32_t n_streams,
                                  const char* path) {
  return guarded([&] {
    need(state && path && (n_streams == 0 || streams), SVL_ERR_INVALID_INPUT, "null argument");
    need(n_streams >= 0, SVL_ERR_INVALID_INPUT, "negative stream count");
    svl::State& s = *state->s;
    svl::check_cuda(cudaSetDevice(s.m->device), "cudaSetDevice");
    svl::voice_load(s, streams, n_streams, path);
  });
}

SVL_API svl_status svl_stt_step(svl_model* model, svl_state* state, int32_t batch,
                                const uint32_t* text_tokens, const uint32_t* audio_tokens,
                                uint32_t* out_tokens, float* out_logits, float* out_extra) {
  return guarded([&] {
    need(model && state && text_tokens && out_tokens, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(m.kind == 0, SVL_ERR_INVALID_INPUT, "not an STT model");
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    const int nq = m.stt.n_q;
    need(nq == 0 || audio_tokens, SVL_ERR_INVALID_INPUT, "null audio tokens");
    // Embedding::forward rejects ids past the table (stt/model.rs:246-250).
    for (int b = 0; b < batch; b++) {
      if (text_tokens[b] > (uint32_t)m.stt.text_card)
        throw Error(SVL_ERR_INVALID_INPUT, "text token out of range");
      for (int c = 0; c < nq; c++)
        if (audio_tokens[b * nq + c] > (uint32_t)m.stt.card)
          throw Error(SVL_ERR_INVALID_INPUT, "audio token out of range");
    }
    check_room(s, batch, 1);
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = m.stream;
    std::memcpy(s.h_tok_in.p, text_tokens, batch * 4);
    if (nq) std::memcpy(s.h_audio_in.p, audio_tokens, (size_t)batch * nq * 4);
    svl::check_cuda(cudaMemcpyAsync(s.tok_in.p, s.h_tok_in.p, batch * 4, cudaMemcpyHostToDevice, st), "h2d");
    if (nq)
      svl::check_cuda(cudaMemcpyAsync(s.audio_in.p, s.h_audio_in.p, (size_t)batch * nq * 4, cudaMemcpyHostToDevice, st), "h2d");
    svl::launch_stt_graph(m, s, batch, st);
    svl::check_cuda(cudaMemcpyAsync(s.h_tok_out.p, s.tok_out.p, batch * 4, cudaMemcpyDeviceToHost, st), "d2h");
    if (out_logits)
      svl::check_cuda(cudaMemcpyAsync(out_logits, s.logits.p, (size_t)batch * m.stt.text_card * 4, cudaMemcpyDeviceToHost, st), "d2h");
    if (out_extra && m.stt.extra_heads_num > 0)
      svl::check_cuda(cudaMemcpyAsync(out_extra, s.extra_p.p, (size_t)batch * m.stt.extra_heads_num * 4, cudaMemcpyDeviceToHost, st), "d2h");
    svl::queue_error_read(s, st);
    svl::check_cuda(cudaStreamSynchronize(st), "step");
    std::memcpy(out_tokens, s.h_tok_out.p, batch * 4);
    for (int b = 0; b < batch; b++) s.hpos[b]++;
    svl::raise_device_error(s, st);
  });
}

SVL_API svl_status svl_stt_step_device(svl_model* model, svl_state* state, int32_t batch,
                                       const uint32_t* d_text_tokens,
                                       const uint32_t* d_audio_tokens, uint32_t* d_out_tokens,
                                       float* d_out_logits, void* cuda_stream) {
  return guarded([&] {
    need(model && state && d_text_tokens && d_out_tokens, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(m.kind == 0, SVL_ERR_INVALID_INPUT, "not an STT model");
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    const int nq = m.stt.n_q;
    need(nq == 0 || d_audio_tokens, SVL_ERR_INVALID_INPUT, "null audio tokens");
    check_room(s, batch, 1);
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : m.stream;
    svl::check_cuda(cudaMemcpyAsync(s.tok_in.p, d_text_tokens, batch * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (nq)
      svl::check_cuda(cudaMemcpyAsync(s.audio_in.p, d_audio_tokens, (size_t)batch * nq * 4, cudaMemcpyDeviceToDevice, st), "copy");
    svl::launch_stt_graph(m, s, batch, st);
    svl::check_cuda(cudaMemcpyAsync(d_out_tokens, s.tok_out.p, batch * 4, cudaMemcpyDeviceToDevice, st), "copy");
    if (d_out_logits)
      svl::check_cuda(cudaMemcpyAsync(d_out_logits, s.logits.p, (size_t)batch * m.stt.text_card * 4, cudaMemcpyDeviceToDevice, st), "copy");
    for (int b = 0; b < batch; b++) s.hpos[b]++;
  });
}

SVL_API svl_status svl_stt_run_frames(svl_model* model, svl_state* state, int32_t batch,
                                      int32_t n_frames, const uint32_t* audio_tokens,
                                      uint32_t* out_tokens) {
  return svl_stt_run_frames_ex(model, state, batch, n_frames, audio_tokens, out_tokens, nullptr);
}

SVL_API svl_status svl_stt_run_frames_ex(svl_model* model, svl_state* state, int32_t batch,
                                         int32_t n_frames, const uint32_t* audio_tokens,
                                         uint32_t* out_tokens, float* out_extra) {
  return guarded([&] {
    need(model && state && out_tokens, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(m.kind == 0, SVL_ERR_INVALID_INPUT, "not an STT model");
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    need(n_frames >= 0, SVL_ERR_INVALID_INPUT, "negative frame count");
    if (n_frames == 0) return;
    const int nq = m.stt.n_q;
    need(nq == 0 || audio_tokens, SVL_ERR_INVALID_INPUT, "null audio tokens");
    check_room(s, batch, n_frames);
    // Recognizer::step (stt/mod.rs:551-565): a stream's first step sees the initial tokens.
    std::vector<uint32_t> audio((size_t)n_frames * batch * nq);
    for (int f = 0; f < n_frames; f++)
      for (int b = 0; b < batch; b++)
        for (int c = 0; c < nq; c++) {
          const size_t i = ((size_t)f * batch + b) * nq + c;
          uint32_t a = audio_tokens[i];
          if (s.hpos[b] + f == 0) a = (uint32_t)m.stt.card;
          if (a > (uint32_t)m.stt.card) throw Error(SVL_ERR_INVALID_INPUT, "audio token out of range");
          audio[i] = a;
        }
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = m.stream;
    const size_t fbytes = (size_t)n_frames * batch * nq * 4, obytes = (size_t)n_frames * batch * 4;
    const int eh = m.stt.extra_heads_num;
    const size_t ebytes = out_extra && eh > 0 ? (size_t)n_frames * batch * eh * 4 : 0;
    if (s.frames_audio.bytes < fbytes) s.frames_audio.alloc(fbytes);
    if (s.frames_out.bytes < obytes) s.frames_out.alloc(obytes);
    if (s.frames_extra.bytes < ebytes) s.frames_extra.alloc(ebytes);
    if (nq) svl::check_cuda(cudaMemcpyAsync(s.frames_audio.p, audio.data(), fbytes, cudaMemcpyHostToDevice, st), "h2d");
    // The text token fed at each stream's next step: text_card at position 0, else the
    // stream's last argmax.
    std::vector<uint32_t> last(batch);
    svl::check_cuda(cudaMemcpyAsync(last.data(), s.tok_out.p, batch * 4, cudaMemcpyDeviceToHost, st), "d2h");
    svl::check_cuda(cudaStreamSynchronize(st), "sync");
    for (int b = 0; b < batch; b++)
      if (s.hpos[b] == 0) last[b] = (uint32_t)m.stt.text_card;
    svl::check_cuda(cudaMemcpyAsync(s.tok_in.p, last.data(), batch * 4, cudaMemcpyHostToDevice, st), "h2d");
    for (int f = 0; f < n_frames; f++) {
      if (nq)
        svl::check_cuda(cudaMemcpyAsync(s.audio_in.p, s.frames_audio.as<uint8_t>() + (size_t)f * batch * nq * 4,
                                        (size_t)batch * nq * 4, cudaMemcpyDeviceToDevice, st), "copy");
      svl::launch_stt_graph(m, s, batch, st);
      svl::check_cuda(cudaMemcpyAsync(s.tok_in.p, s.tok_out.p, batch * 4, cudaMemcpyDeviceToDevice, st), "copy");
      svl::check_cuda(cudaMemcpyAsync(s.frames_out.as<uint8_t>() + (size_t)f * batch * 4, s.tok_out.p, batch * 4,
                                      cudaMemcpyDeviceToDevice, st), "copy");
      if (ebytes)
        svl::check_cuda(cudaMemcpyAsync(s.frames_extra.as<uint8_t>() + (size_t)f * batch * eh * 4, s.extra_p.p,
                                        (size_t)batch * eh * 4, cudaMemcpyDeviceToDevice, st), "copy");
    }
    svl::check_cuda(cudaMemcpyAsync(out_tokens, s.frames_out.p, obytes, cudaMemcpyDeviceToHost, st), "d2h");
    if (ebytes) svl::check_cuda(cudaMemcpyAsync(out_extra, s.frames_extra.p, ebytes, cudaMemcpyDeviceToHost, st), "d2h");
    svl::queue_error_read(s, st);
    svl::check_cuda(cudaStreamSynchronize(st), "frames");
    for (int b = 0; b < batch; b++) s.hpos[b] += n_frames;
    svl::raise_device_error(s, st);
  });
}

SVL_API svl_status svl_transformer_forward(svl_model* model, svl_state* state, int32_t stream,
                                           float* xs, int32_t t) {
  return guarded([&] {
    need(model && state && xs, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    check_stream(s, stream);
    need(t >= 1, SVL_ERR_INVALID_INPUT, "t must be positive");
    check_room(s, stream, 1, t);
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = m.stream;
    const int d = m.cfg.d_model;
    float* xrow = s.x.as<float>() + (int64_t)stream * d;
    // Causal attention makes a block of t queries equal to t single steps
    // (streaming_matches_full_sequence, nn/transformer.rs:598-628).
    for (int i = 0; i < t; i++) {
      svl::check_cuda(cudaMemcpyAsync(xrow, xs + (int64_t)i * d, d * 4, cudaMemcpyHostToDevice, st), "h2d");
      svl::enqueue_layers(m, s, stream, 1, st);
      svl::launch_advance_positions(s.pos.as<int>() + stream, 1, st);
      svl::check_cuda(cudaMemcpyAsync(xs + (int64_t)i * d, xrow, d * 4, cudaMemcpyDeviceToHost, st), "d2h");
    }
    svl::check_cuda(cudaStreamSynchronize(st), "forward");
    s.hpos[stream] += t;
  });
}

SVL_API svl_status svl_profile_kernels(svl_model* model, svl_state* state, int32_t batch,
                                       int32_t which, int32_t iters, void* cuda_stream,
                                       int64_t* bytes_per_iter) {
  return guarded([&] {
    need(model && state, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    need(which == 0 || which == 1 || (which == 2 && m.kind == 1), SVL_ERR_INVALID_INPUT,
         "which must be 0 or 1 (2: the flow head of a TTS model)");
    need(iters >= 0, SVL_ERR_INVALID_INPUT, "negative iters");
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : m.stream;
    int64_t bytes = 0;
    for (int i = 0; i < iters; i++) bytes = svl::enqueue_profile(m, s, batch, which, st);
    if (iters == 0) {
      // Bytes only: enqueue nothing.
      bytes = 0;
    }
    if (bytes_per_iter) *bytes_per_iter = bytes;
    svl::check_cuda(cudaGetLastError(), "profile launch");
  });
}

SVL_API svl_status svl_state_error(svl_state* state) {
  return guarded([&] {
    need(state, SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    svl::check_cuda(cudaSetDevice(s.m->device), "cudaSetDevice");
    svl::check_cuda(cudaDeviceSynchronize(), "sync");
    svl::queue_error_read(s, s.m->stream);
    svl::check_cuda(cudaStreamSynchronize(s.m->stream), "sync");
    svl::raise_device_error(s, s.m->stream);
  });
}

SVL_API svl_status svl_step_kernel_count(svl_model* model, svl_state* state, int32_t batch,
                                         int32_t* kernels) {
  return guarded([&] {
    need(model && state && kernels, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    *kernels = m.kind == 0 ? svl::capture_stt_graph(m, s, batch, m.stream)
                           : svl::capture_tts_graph(m, s, batch, 1, m.stream);
  });
}

namespace {

// FlowLm::prompt_text for streams [b0, b0 + nb), n tokens each (host tokens [nb][n]).
void tts_prompt(svl::Model& m, svl::State& s, int b0, int nb, const uint32_t* tokens, int n) {
  need(m.kind == 1, SVL_ERR_INVALID_INPUT, "not a TTS model");
  need(tokens && n >= 1, SVL_ERR_INVALID_INPUT, "no tokens");
  for (int64_t i = 0; i < (int64_t)nb * n; i++)
    if (tokens[i] > (uint32_t)m.tts.text_bins)
      throw Error(SVL_ERR_INVALID_INPUT, "text token " + std::to_string(tokens[i]) + " out of range");
  check_room(s, b0, nb, n);
  svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
  cudaStream_t st = m.stream;
  const size_t bytes = (size_t)nb * n * 4;
  if (s.prompt_tok.bytes < bytes) {
    svl::check_cuda(cudaStreamSynchronize(st), "sync");
    s.prompt_tok.alloc(bytes);
  }
  svl::check_cuda(cudaMemcpyAsync(s.prompt_tok.p, tokens, bytes, cudaMemcpyHostToDevice, st), "h2d");
  svl::enqueue_tts_prompt(m, s, b0, nb, s.prompt_tok.as<uint32_t>(), n, st);
  svl::check_cuda(cudaStreamSynchronize(st), "prompt");
  for (int b = b0; b < b0 + nb; b++) s.hpos[b] += n;
}

}  // namespace

SVL_API svl_status svl_tts_prompt_text(svl_model* model, svl_state* state, int32_t stream,
                                       const uint32_t* tokens, int32_t n) {
  return guarded([&] {
    need(model && state, SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    need(s.m == model->m, SVL_ERR_INVALID_INPUT, "state of another model");
    check_stream(s, stream);
    tts_prompt(*model->m, s, stream, 1, tokens, n);
  });
}

SVL_API svl_status svl_tts_prompt_text_batch(svl_model* model, svl_state* state, int32_t batch,
                                             const uint32_t* tokens, int32_t n) {
  return guarded([&] {
    need(model && state, SVL_ERR_INVALID_INPUT, "null argument");
    svl::State& s = *state->s;
    need(s.m == model->m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    tts_prompt(*model->m, s, 0, batch, tokens, n);
  });
}

SVL_API svl_status svl_tts_step_device(svl_model* model, svl_state* state, int32_t batch,
                                       const float* d_latent_in, const float* d_noise,
                                       int32_t decode_steps, float* d_latent_out, float* d_eos,
                                       void* cuda_stream) {
  return guarded([&] {
    need(model && state && d_noise && d_latent_out && d_eos, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(m.kind == 1, SVL_ERR_INVALID_INPUT, "not a TTS model");
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    const int steps = decode_steps < 1 ? 1 : decode_steps;
    need(steps <= 64, SVL_ERR_INVALID_INPUT, "decode_steps above 64");
    check_room(s, batch, 1);
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : m.stream;
    const size_t row = (size_t)m.tts.latent_dim * 4;
    if (d_latent_in) {
      svl::check_cuda(cudaMemcpyAsync(s.latent_in.p, d_latent_in, row * batch, cudaMemcpyDeviceToDevice, st), "copy");
    } else {
      for (int b = 0; b < batch; b++)
        svl::check_cuda(cudaMemcpyAsync(s.latent_in.as<uint8_t>() + row * b, m.bos.p, row,
                                        cudaMemcpyDeviceToDevice, st), "bos");
    }
    svl::check_cuda(cudaMemcpyAsync(s.noise.p, d_noise, row * batch, cudaMemcpyDeviceToDevice, st), "copy");
    svl::launch_tts_graph(m, s, batch, steps, st);
    svl::check_cuda(cudaMemcpyAsync(d_latent_out, s.latent_out.p, row * batch, cudaMemcpyDeviceToDevice, st), "copy");
    svl::check_cuda(cudaMemcpyAsync(d_eos, s.eos.p, (size_t)batch * 4, cudaMemcpyDeviceToDevice, st), "copy");
    for (int b = 0; b < batch; b++) s.hpos[b]++;
  });
}

SVL_API svl_status svl_tts_step(svl_model* model, svl_state* state, int32_t batch,
                                const float* latent_in, const float* noise, int32_t decode_steps,
                                float* latent_out, float* eos_logit) {
  return guarded([&] {
    need(model && state && noise && latent_out && eos_logit, SVL_ERR_INVALID_INPUT, "null argument");
    svl::Model& m = *model->m;
    svl::State& s = *state->s;
    need(m.kind == 1, SVL_ERR_INVALID_INPUT, "not a TTS model");
    need(s.m == &m, SVL_ERR_INVALID_INPUT, "state of another model");
    need(batch >= 1 && batch <= s.max_batch, SVL_ERR_INVALID_INPUT, "batch out of range");
    const int steps = decode_steps < 1 ? 1 : decode_steps;  // FlowHead::decode runs >= 1 step
    need(steps <= 64, SVL_ERR_INVALID_INPUT, "decode_steps above 64");
    check_room(s, batch, 1);
    svl::check_cuda(cudaSetDevice(m.device), "cudaSetDevice");
    cudaStream_t st = m.stream;
    const int lat = m.tts.latent_dim;
    const size_t row = (size_t)lat * 4;
    if (latent_in) {
      svl::check_cuda(cudaMemcpyAsync(s.latent_in.p, latent_in, row * batch, cudaMemcpyHostToDevice, st), "h2d");
    } else {
      // BOS for every stream (FlowLm::step with previous = None, flow_lm.rs:167-170).
      for (int b = 0; b < batch; b++)
        svl::check_cuda(cudaMemcpyAsync(s.latent_in.as<uint8_t>() + row * b, m.bos.p, row,
                                        cudaMemcpyDeviceToDevice, st), "bos");
    }
    svl::check_cuda(cudaMemcpyAsync(s.noise.p, noise, row * batch, cudaMemcpyHostToDevice, st), "h2d");
    svl::launch_tts_graph(m, s, batch, steps, st);
    svl::check_cuda(cudaMemcpyAsync(latent_out, s.latent_out.p, row * batch, cudaMemcpyDeviceToHost, st), "d2h");
    svl::check_cuda(cudaMemcpyAsync(eos_logit, s.eos.p, (size_t)batch * 4, cudaMemcpyDeviceToHost, st), "d2h");
    svl::queue_error_read(s, st);
    svl::check_cuda(cudaStreamSynchronize(st), "tts step");
    for (int b = 0; b < batch; b++) s.hpos[b] += 1;
    svl::raise_device_error(s, st);
  });
}

}  // extern "C"
