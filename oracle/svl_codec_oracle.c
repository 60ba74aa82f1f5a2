/*
 * svl_codec_oracle.c — CPU restatement of semantic-voice-local's Mimi codec (SEANet encoder and
 * decoder, the projected transformers, learnt resampling) and Kyutai STT's split residual
 * vector quantizer.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the codec kernels. Only tests/ and
 * bench.py's CPU legs load it (as part of libsvl_oracle.so); the product never links it.
 *
 * Follows, for one stream:
 *  - StreamingConv1d::forward (nn/conv.rs:122-179) with im2col (nn/kernels/conv.rs:8-85):
 *    the carried-over context, constant / replicate padding of the first chunk, output l =
 *    sum over (channel c, tap j) of w[o][c][j] x[l stride + j dil], then + bias; the sum is
 *    blocked in chunks of floor(1024 / k) channels (FMA chains, then the chunks' sums in order);
 *  - StreamingConvTranspose1d::forward_taps (nn/conv.rs:296-323) with overlap_add
 *    (nn/kernels/conv.rs:87-166): bias on the complete outputs, + the previous partial, + the
 *    taps in tap order; the tail becomes the next partial;
 *  - ResnetBlock / SeanetEncoder / SeanetDecoder (nn/seanet.rs:36-245), ELU
 *    (nn/kernels/activation.rs:60-67);
 *  - ProjectedTransformer (nn/mimi.rs:66-123) through orc_transformer_create;
 *  - MimiEncoder::encode_step / MimiDecoder::decode_step (nn/mimi.rs:184-271);
 *  - Quantizer / ResidualQuantizer / Codebook (stt/model.rs:84-170).
 *
 * Parity status: the products inside candle's matmul (gemm crate, blocked) have an order of
 * their own; this file sums each output in fixed chunks of im2col columns (one FMA chain each), so
 * against candle the convolutions and distances are "parity unpinned" (tolerance-level), while
 * the streaming semantics (context, padding, overlap-add order, argmin ties) follow the source.
 * The reference's own tests for these pieces (streaming equals one pass, conv vs direct
 * convolution, transposed conv vs candle) are restated in tests/test_codec_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "svl_oracle.h"

/* ------------------------------------------------------------------ streaming convolutions */

static int conv_ctx(int k, int stride, int dil) {
  int c = (k - 1) * dil + 1 - stride;
  return c > 0 ? c : 0;
}

int orc_conv1d_stream(int cin, int cout, int k, int stride, int dil, int replicate, const float* w,
                      const float* bias, float* prev, int* started, const float* x, int t, int elu,
                      const float* skip, float* out) {
  if (t <= 0 || t % stride) return -1;
  const int ctx = conv_ctx(k, stride, dil), total = ctx + t, len = t / stride;
  float* xc = (float*)malloc(sizeof(float) * (size_t)cin * total);
  for (int c = 0; c < cin; c++) {
    for (int i = 0; i < ctx; i++) {
      float v;
      if (*started) v = prev[(size_t)c * ctx + i];
      else if (replicate) v = elu ? orc_elu(x[(size_t)c * t]) : x[(size_t)c * t];
      else v = 0.0f;
      xc[(size_t)c * total + i] = v;
    }
    for (int i = 0; i < t; i++) {
      float v = x[(size_t)c * t + i];
      xc[(size_t)c * total + ctx + i] = elu ? orc_elu(v) : v;
    }
  }
  /* Chunks of floor(1024 / k) input channels: each an FMA chain from zero over its (channel,
   * tap) terms in order, the chunks' sums then added in order (a fixed blocking of the
   * reduction, as a blocked matmul has; it depends on the layer's shape only). */
  const int cpc = 1024 / k > 0 ? 1024 / k : 1;
  for (int o = 0; o < cout; o++)
    for (int l = 0; l < len; l++) {
      float v = 0.0f;
      for (int c0 = 0; c0 < cin; c0 += cpc) {
        float acc = 0.0f;
        const int c1 = c0 + cpc < cin ? c0 + cpc : cin;
        for (int c = c0; c < c1; c++)
          for (int j = 0; j < k; j++)
            acc = fmaf(w[((size_t)o * cin + c) * k + j], xc[(size_t)c * total + (size_t)l * stride + (size_t)j * dil], acc);
        v = c0 == 0 ? acc : v + acc;
      }
      if (bias) v = v + bias[o];
      if (skip) v = skip[(size_t)o * len + l] + v;
      out[(size_t)o * len + l] = v;
    }
  for (int c = 0; c < cin; c++)
    for (int u = 0; u < ctx; u++) prev[(size_t)c * ctx + u] = xc[(size_t)c * total + t + u];
  *started = 1;
  free(xc);
  return 0;
}

int orc_convtr1d_stream(int cin, int cout, int k, int stride, int depthwise, const float* w,
                        const float* bias, float* partial, const float* x, int t, int elu,
                        float* out) {
  if (t <= 0 || k < stride) return -1;
  const int overlap = k - stride, complete = t * stride, total = complete + overlap;
  float* xa = (float*)malloc(sizeof(float) * (size_t)cin * t);
  for (size_t i = 0; i < (size_t)cin * t; i++) xa[i] = elu ? orc_elu(x[i]) : x[i];
  float* tail = (float*)malloc(sizeof(float) * (size_t)cout * (overlap > 0 ? overlap : 1));
  for (int o = 0; o < cout; o++)
    for (int s = 0; s < total; s++) {
      float v = (s < complete && bias) ? bias[o] : 0.0f;
      if (s < overlap) v = v + partial[(size_t)o * overlap + s];
      for (int h = 0;; h++) {
        int tap = s % stride + h * stride, step = s / stride - h;
        if (tap >= k) break;
        if (step < 0 || step >= t) continue;
        float p;
        if (depthwise) {
          p = w[(size_t)o * k + tap] * xa[(size_t)o * t + step];
        } else {
          /* The taps' products are a 1x1 convolution: chunks of 1024 input channels. */
          p = 0.0f;
          for (int c0 = 0; c0 < cin; c0 += 1024) {
            float acc = 0.0f;
            const int c1 = c0 + 1024 < cin ? c0 + 1024 : cin;
            for (int c = c0; c < c1; c++) acc = fmaf(w[((size_t)c * cout + o) * k + tap], xa[(size_t)c * t + step], acc);
            p = c0 == 0 ? acc : p + acc;
          }
        }
        v = v + p;
      }
      if (s < complete) out[(size_t)o * complete + s] = v;
      else tail[(size_t)o * overlap + (s - complete)] = v;
    }
  if (overlap > 0) memcpy(partial, tail, sizeof(float) * (size_t)cout * overlap);
  free(tail);
  free(xa);
  return 0;
}

/* ------------------------------------------------------------------ Mimi */

typedef struct {
  int tr, depthwise, cin, cout, k, stride, dil, replicate;
  const float *w, *bias; /* borrowed from the caller's tensors */
} oconv;
enum { OB_IN = 0, OB_A = 1, OB_B = 2, OB_H = 3, OB_OUT = 4 };
typedef struct {
  int layer, in, out, elu, skip;
} ostep;

struct orc_mimi {
  orc_mimi_cfg cfg;
  int frame_size, enc_stride, dec_stride;
  oconv* convs;
  int n_convs, cap_convs;
  ostep *enc, *dec;
  int n_enc, n_dec;
  int down, up, enc_in, enc_out, dec_in, dec_out;
  int latent_proj, latent_dim; /* Tts::decode_latent's quantizer.output_proj (tts/mod.rs:218-224) */
  orc_lm *enc_tr, *dec_tr;
  float* owned_w[64];
  int n_owned;
};

struct orc_mimi_state {
  orc_mimi* m;
  float** st;  /* per conv layer: prev [cin][ctx] or partial [cout][overlap] */
  int enc_started, dec_started;
  orc_state *enc_ts, *dec_ts;
};

static const orc_tensor* cfind(const orc_tensor* t, int n, const char* name) {
  for (int i = 0; i < n; i++)
    if (t[i].name && !strcmp(t[i].name, name)) return &t[i];
  return NULL;
}
static const float* cget(const orc_tensor* t, int n, const char* name, int64_t numel, int* ok) {
  const orc_tensor* v = cfind(t, n, name);
  if (!v || v->numel != numel || !v->data) {
    fprintf(stderr, "codec oracle: tensor %s missing or of the wrong size\n", name);
    *ok = 0;
    return NULL;
  }
  return v->data;
}

static int new_slot(orc_mimi* m) {
  if (m->n_convs == m->cap_convs) {
    m->cap_convs = m->cap_convs ? 2 * m->cap_convs : 32;
    m->convs = (oconv*)realloc(m->convs, sizeof(oconv) * (size_t)m->cap_convs);
  }
  memset(&m->convs[m->n_convs], 0, sizeof(oconv));
  return m->n_convs++;
}
static int add_conv(orc_mimi* m, const orc_tensor* t, int n, const char* prefix, int cin, int cout, int k,
                    int stride, int dil, int replicate, int bias, int* ok) {
  const int idx = new_slot(m);
  oconv* L = &m->convs[idx];
  L->cin = cin;
  L->cout = cout;
  L->k = k;
  L->stride = stride;
  L->dil = dil;
  L->replicate = replicate;
  char nm[320];
  snprintf(nm, sizeof nm, "%s.weight", prefix);
  L->w = cget(t, n, nm, (int64_t)cout * cin * k, ok);
  if (bias) {
    snprintf(nm, sizeof nm, "%s.bias", prefix);
    L->bias = cget(t, n, nm, cout, ok);
  }
  return idx;
}
static int add_convtr(orc_mimi* m, const orc_tensor* t, int n, const char* prefix, int cin, int cout, int k,
                      int stride, int groups, int bias, int* ok) {
  const int i = new_slot(m);
  oconv* L = &m->convs[i];
  L->tr = 1;
  L->depthwise = groups != 1;
  L->cin = cin;
  L->cout = cout;
  L->k = k;
  L->stride = stride;
  char nm[320];
  snprintf(nm, sizeof nm, "%s.weight", prefix);
  L->w = cget(t, n, nm, (int64_t)cin * (cout / groups) * k, ok);
  L->bias = NULL;
  if (bias) {
    snprintf(nm, sizeof nm, "%s.bias", prefix);
    L->bias = cget(t, n, nm, cout, ok);
  }
  return i;
}
static void push_step(ostep** v, int* nv, int layer, int in, int out, int elu, int skip) {
  *v = (ostep*)realloc(*v, sizeof(ostep) * (size_t)(*nv + 1));
  (*v)[*nv] = (ostep){layer, in, out, elu, skip};
  (*nv)++;
}
static void add_resnet(orc_mimi* m, const orc_tensor* t, int n, ostep** v, int* nv, const orc_seanet_cfg* s,
                       int idx, const char* part, int dim, int dil, int buf, int* ok) {
  char nm[256];
  int hidden = dim / s->compress;
  snprintf(nm, sizeof nm, "%s.model.%d.block.1.conv", part, idx);
  int a = add_conv(m, t, n, nm, dim, hidden, s->residual_kernel_size, 1, dil, s->pad_mode, 1, ok);
  snprintf(nm, sizeof nm, "%s.model.%d.block.3.conv", part, idx);
  int b = add_conv(m, t, n, nm, hidden, dim, 1, 1, 1, s->pad_mode, 1, ok);
  push_step(v, nv, a, buf, OB_H, 1, -1);
  push_step(v, nv, b, OB_H, buf, 1, buf);
}

static int hop(const orc_seanet_cfg* s) {
  int h = 1;
  for (int i = 0; i < s->n_ratios; i++) h *= s->ratios[i];
  return h;
}

static orc_tcfg tr_cfg(const orc_ptrans_cfg* p, int exact) {
  orc_tcfg c;
  memset(&c, 0, sizeof c);
  c.d_model = p->d_model;
  c.num_layers = p->num_layers;
  c.num_heads = p->num_heads;
  c.num_kv_heads = p->num_heads;
  c.head_dim = p->d_model / p->num_heads;
  c.ffn_kind = exact ? 1 : 0;
  c.ffn_hidden = p->dim_feedforward;
  c.norm_kind = 0;
  c.norm_eps = 1e-5f;
  c.layer_scale = 1;
  c.context = p->context;
  c.weight_dtype = 0;
  c.kv_dtype = 0;
  c.max_period = p->max_period;
  return c;
}

orc_mimi* orc_mimi_create(const orc_mimi_cfg* cfg, const orc_tensor* t, int n) {
  orc_mimi* m = (orc_mimi*)calloc(1, sizeof(orc_mimi));
  m->cfg = *cfg;
  m->down = m->up = m->enc_in = m->enc_out = m->dec_in = m->dec_out = m->latent_proj = -1;
  m->frame_size = (int)lround((double)cfg->sample_rate / cfg->frame_rate);
  int ok = 1;
  char nm[256];
  if (cfg->parts & 1) {
    const orc_seanet_cfg* s = &cfg->encoder;
    m->enc_stride = (int)lround((double)cfg->sample_rate / hop(s) / cfg->frame_rate);
    int li = 0, cur = OB_A, mult = 1;
    snprintf(nm, sizeof nm, "encoder.model.%d.conv", li++);
    int c0 = add_conv(m, t, n, nm, s->channels, s->n_filters, s->kernel_size, 1, 1, s->pad_mode, 1, &ok);
    push_step(&m->enc, &m->n_enc, c0, OB_IN, OB_A, 0, -1);
    for (int r = s->n_ratios - 1; r >= 0; r--) {
      int dim = mult * s->n_filters, dil = 1;
      for (int j = 0; j < s->n_residual_layers; j++, dil *= s->dilation_base)
        add_resnet(m, t, n, &m->enc, &m->n_enc, s, li++, "encoder", dim, dil, cur, &ok);
      li++; /* Elu */
      int nxt = cur == OB_A ? OB_B : OB_A;
      snprintf(nm, sizeof nm, "encoder.model.%d.conv", li++);
      int dc = add_conv(m, t, n, nm, dim, 2 * dim, 2 * s->ratios[r], s->ratios[r], 1, s->pad_mode, 1, &ok);
      push_step(&m->enc, &m->n_enc, dc, cur, nxt, 1, -1);
      cur = nxt;
      mult *= 2;
    }
    li++; /* Elu */
    snprintf(nm, sizeof nm, "encoder.model.%d.conv", li);
    int last = add_conv(m, t, n, nm, mult * s->n_filters, s->dimension, s->last_kernel_size, 1, 1, s->pad_mode, 1, &ok);
    push_step(&m->enc, &m->n_enc, last, cur, OB_OUT, 1, -1);
    const orc_ptrans_cfg* p = &cfg->encoder_transformer;
    if (p->input_dimension != p->d_model)
      m->enc_in = add_conv(m, t, n, "encoder_transformer.input_proj", p->input_dimension, p->d_model, 1, 1, 1, 0, 0, &ok);
    if (p->output_dimension != p->d_model)
      m->enc_out = add_conv(m, t, n, "encoder_transformer.output_projs.0", p->d_model, p->output_dimension, 1, 1, 1, 0, 0, &ok);
    orc_tcfg tc = tr_cfg(p, cfg->exact_gelu);
    m->enc_tr = orc_transformer_create(&tc, "encoder_transformer.transformer.", t, n);
    if (!m->enc_tr) ok = 0;
    if (m->enc_stride > 1)
      m->down = add_conv(m, t, n, "downsample.conv.conv", p->output_dimension, cfg->inner_dim, 2 * m->enc_stride,
                         m->enc_stride, 1, 1, 0, &ok);
  }
  if (cfg->parts & 2) {
    const orc_seanet_cfg* s = &cfg->decoder;
    m->dec_stride = (int)lround((double)cfg->sample_rate / hop(s) / cfg->frame_rate);
    const orc_ptrans_cfg* p = &cfg->decoder_transformer;
    if (m->dec_stride > 1) {
      int i = add_convtr(m, t, n, "upsample.convtr.convtr", cfg->outer_dim, s->dimension, 2 * m->dec_stride,
                         m->dec_stride, s->dimension, 0, &ok);
      m->up = i;
    }
    if (p->input_dimension != p->d_model)
      m->dec_in = add_conv(m, t, n, "decoder_transformer.input_proj", p->input_dimension, p->d_model, 1, 1, 1, 0, 0, &ok);
    if (p->output_dimension != p->d_model)
      m->dec_out = add_conv(m, t, n, "decoder_transformer.output_projs.0", p->d_model, p->output_dimension, 1, 1, 1, 0, 0, &ok);
    orc_tcfg tc = tr_cfg(p, cfg->exact_gelu);
    m->dec_tr = orc_transformer_create(&tc, "decoder_transformer.transformer.", t, n);
    if (!m->dec_tr) ok = 0;
    const orc_tensor* lp = cfind(t, n, "quantizer.output_proj.weight");
    if (lp && lp->numel > 0 && lp->numel % cfg->outer_dim == 0) {
      m->latent_dim = (int)(lp->numel / cfg->outer_dim);
      m->latent_proj = add_conv(m, t, n, "quantizer.output_proj", m->latent_dim, cfg->outer_dim, 1, 1, 1, 0, 0, &ok);
    }
    int mult = 1 << s->n_ratios, li = 0, cur = OB_A;
    snprintf(nm, sizeof nm, "decoder.model.%d.conv", li++);
    int c0 = add_conv(m, t, n, nm, s->dimension, mult * s->n_filters, s->kernel_size, 1, 1, s->pad_mode, 1, &ok);
    push_step(&m->dec, &m->n_dec, c0, OB_IN, OB_A, 0, -1);
    for (int r = 0; r < s->n_ratios; r++) {
      int dim = mult * s->n_filters, dil = 1;
      li++; /* Elu */
      int nxt = cur == OB_A ? OB_B : OB_A;
      snprintf(nm, sizeof nm, "decoder.model.%d.convtr", li++);
      int up = add_convtr(m, t, n, nm, dim, dim / 2, 2 * s->ratios[r], s->ratios[r], 1, 1, &ok);
      push_step(&m->dec, &m->n_dec, up, cur, nxt, 1, -1);
      cur = nxt;
      for (int j = 0; j < s->n_residual_layers; j++, dil *= s->dilation_base)
        add_resnet(m, t, n, &m->dec, &m->n_dec, s, li++, "decoder", dim / 2, dil, cur, &ok);
      mult /= 2;
    }
    li++; /* Elu */
    snprintf(nm, sizeof nm, "decoder.model.%d.conv", li);
    int last = add_conv(m, t, n, nm, s->n_filters, s->channels, s->last_kernel_size, 1, 1, s->pad_mode, 1, &ok);
    push_step(&m->dec, &m->n_dec, last, cur, OB_OUT, 1, -1);
  }
  if (!ok) {
    orc_mimi_free(m);
    return NULL;
  }
  return m;
}

void orc_mimi_free(orc_mimi* m) {
  if (!m) return;
  free(m->convs);
  free(m->enc);
  free(m->dec);
  orc_lm_free(m->enc_tr);
  orc_lm_free(m->dec_tr);
  free(m);
}

int orc_mimi_frame_size(const orc_mimi* m) { return m->frame_size; }

orc_mimi_state* orc_mimi_state_create(orc_mimi* m) {
  orc_mimi_state* s = (orc_mimi_state*)calloc(1, sizeof(orc_mimi_state));
  s->m = m;
  s->st = (float**)calloc((size_t)(m->n_convs ? m->n_convs : 1), sizeof(float*));
  for (int i = 0; i < m->n_convs; i++) {
    const oconv* L = &m->convs[i];
    size_t n = L->tr ? (size_t)L->cout * (L->k - L->stride) : (size_t)L->cin * conv_ctx(L->k, L->stride, L->dil);
    s->st[i] = (float*)calloc(n ? n : 1, sizeof(float));
  }
  if (m->enc_tr) s->enc_ts = orc_state_create(m->enc_tr);
  if (m->dec_tr) s->dec_ts = orc_state_create(m->dec_tr);
  return s;
}

void orc_mimi_state_free(orc_mimi_state* s) {
  if (!s) return;
  for (int i = 0; i < s->m->n_convs; i++) free(s->st[i]);
  free(s->st);
  orc_state_free(s->enc_ts);
  orc_state_free(s->dec_ts);
  free(s);
}

typedef struct {
  float* p;
  int C, t;
} oview;

/* One layer on a packed [C][t] block; the result is a new block (the caller frees it). */
static oview run_layer(orc_mimi_state* S, int li, oview in, int elu, const oview* skip, int* started) {
  const oconv* L = &S->m->convs[li];
  oview out;
  out.C = L->cout;
  out.t = L->tr ? in.t * L->stride : in.t / L->stride;
  out.p = (float*)malloc(sizeof(float) * (size_t)out.C * (out.t ? out.t : 1));
  if (L->tr)
    orc_convtr1d_stream(L->cin, L->cout, L->k, L->stride, L->depthwise, L->w, L->bias, S->st[li], in.p, in.t, elu, out.p);
  else {
    int st = *started; /* every convolution of one call sees the same "first chunk" flag */
    orc_conv1d_stream(L->cin, L->cout, L->k, L->stride, L->dil, L->replicate, L->w, L->bias, S->st[li], &st, in.p,
                      in.t, elu, skip ? skip->p : NULL, out.p);
  }
  return out;
}

static oview run_seanet(orc_mimi_state* S, const ostep* steps, int n, oview in, int* started) {
  oview v[5] = {{0, 0, 0}};
  v[OB_IN] = in;
  oview last = in;
  float** made = (float**)malloc(sizeof(float*) * (size_t)(n ? n : 1));
  for (int i = 0; i < n; i++) {
    const ostep* s = &steps[i];
    const oview* skip = s->skip >= 0 ? &v[s->skip] : NULL;
    last = run_layer(S, s->layer, v[s->in], s->elu, skip, started);
    made[i] = last.p;
    v[s->out] = last;
  }
  for (int i = 0; i < n; i++)
    if (made[i] != last.p) free(made[i]);
  free(made);
  return last;
}

/* Transformer::forward over the t frames of a [C][t] block, in place. */
static void run_transformer(orc_lm* tr, orc_state* ts, oview x) {
  float* rows = (float*)malloc(sizeof(float) * (size_t)x.C * x.t);
  for (int c = 0; c < x.C; c++)
    for (int i = 0; i < x.t; i++) rows[(size_t)i * x.C + c] = x.p[(size_t)c * x.t + i];
  orc_transformer_forward(tr, ts, rows, x.t);
  for (int c = 0; c < x.C; c++)
    for (int i = 0; i < x.t; i++) x.p[(size_t)c * x.t + i] = rows[(size_t)i * x.C + c];
  free(rows);
}

static oview layer_owned(orc_mimi_state* S, int li, oview in, int* started) {
  oview o = run_layer(S, li, in, 0, NULL, started);
  return o;
}

int orc_mimi_encode_step(orc_mimi* m, orc_mimi_state* S, const float* pcm, int frames, float* latent) {
  if (!m->enc_tr || frames <= 0) return -1;
  oview in = {(float*)pcm, m->cfg.encoder.channels, frames * m->frame_size};
  oview x = run_seanet(S, m->enc, m->n_enc, in, &S->enc_started);
  if (m->enc_in >= 0) {
    oview y = layer_owned(S, m->enc_in, x, &S->enc_started);
    free(x.p);
    x = y;
  }
  run_transformer(m->enc_tr, S->enc_ts, x);
  if (m->enc_out >= 0) {
    oview y = layer_owned(S, m->enc_out, x, &S->enc_started);
    free(x.p);
    x = y;
  }
  if (m->down >= 0) {
    oview y = layer_owned(S, m->down, x, &S->enc_started);
    free(x.p);
    x = y;
  }
  memcpy(latent, x.p, sizeof(float) * (size_t)x.C * x.t);
  free(x.p);
  S->enc_started = 1;
  return 0;
}

int orc_mimi_decode_step(orc_mimi* m, orc_mimi_state* S, const float* latent, int frames, float* pcm) {
  if (!m->dec_tr || frames <= 0) return -1;
  oview in = {(float*)latent, m->cfg.outer_dim, frames};
  oview x;
  if (m->up >= 0) {
    x = layer_owned(S, m->up, in, &S->dec_started);
  } else {
    x.C = in.C;
    x.t = in.t;
    x.p = (float*)malloc(sizeof(float) * (size_t)in.C * in.t);
    memcpy(x.p, latent, sizeof(float) * (size_t)in.C * in.t);
  }
  if (m->dec_in >= 0) {
    oview y = layer_owned(S, m->dec_in, x, &S->dec_started);
    free(x.p);
    x = y;
  }
  run_transformer(m->dec_tr, S->dec_ts, x);
  if (m->dec_out >= 0) {
    oview y = layer_owned(S, m->dec_out, x, &S->dec_started);
    free(x.p);
    x = y;
  }
  oview y = run_seanet(S, m->dec, m->n_dec, x, &S->dec_started);
  memcpy(pcm, y.p, sizeof(float) * (size_t)y.C * y.t);
  free(y.p);
  free(x.p);
  S->dec_started = 1;
  return 0;
}

/* Tts::decode_latent (tts/mod.rs:441-447): latent [frames][latent_dim] times emb_std plus
 * emb_mean (both NULL: as is), the latent projection, then MimiDecoder::decode_step. */
int orc_mimi_decode_latent(orc_mimi* m, orc_mimi_state* S, const float* latent, int frames,
                           const float* emb_std, const float* emb_mean, float* pcm) {
  if (m->latent_proj < 0 || frames <= 0) return -1;
  const oconv* L = &m->convs[m->latent_proj];
  float* x = (float*)malloc(sizeof(float) * (size_t)L->cin * frames);
  for (int c = 0; c < L->cin; c++)
    for (int f = 0; f < frames; f++) {
      float v = latent[(size_t)f * L->cin + c];
      if (emb_std) v = v * emb_std[c] + emb_mean[c];
      x[(size_t)c * frames + f] = v;
    }
  oview in = {x, L->cin, frames};
  int started = 1;
  oview y = run_layer(S, m->latent_proj, in, 0, NULL, &started);
  int rc = orc_mimi_decode_step(m, S, y.p, frames, pcm);
  free(y.p);
  free(x);
  return rc;
}

/* ------------------------------------------------------------------ residual vector quantizer */

#define RVQ_DIM 256 /* ResidualQuantizer::DIM */
#define RVQ_IN 512

struct orc_rvq {
  int n_q, bins;
  float* proj[2]; /* [256][512] */
  float* emb;     /* [n_q][bins][256] */
  float* hn;      /* [n_q][bins] */
};

orc_rvq* orc_rvq_create(int n_q, int bins, const orc_tensor* t, int n) {
  if (n_q < 1 || bins < 1) return NULL;
  orc_rvq* q = (orc_rvq*)calloc(1, sizeof(orc_rvq));
  q->n_q = n_q;
  q->bins = bins;
  int ok = 1;
  const char* parts[2] = {"quantizer.rvq_first", "quantizer.rvq_rest"};
  char nm[256];
  for (int p = 0; p < 2 && ok; p++) {
    if (p == 1 && n_q == 1) break;
    snprintf(nm, sizeof nm, "%s.input_proj.weight", parts[p]);
    const float* w = cget(t, n, nm, (int64_t)RVQ_DIM * RVQ_IN, &ok);
    if (!ok) break;
    q->proj[p] = (float*)malloc(sizeof(float) * RVQ_DIM * RVQ_IN);
    memcpy(q->proj[p], w, sizeof(float) * RVQ_DIM * RVQ_IN);
  }
  q->emb = (float*)malloc(sizeof(float) * (size_t)n_q * bins * RVQ_DIM);
  q->hn = (float*)malloc(sizeof(float) * (size_t)n_q * bins);
  for (int k = 0; k < n_q && ok; k++) {
    char pre[200];
    if (k == 0) snprintf(pre, sizeof pre, "%s.vq.layers.0._codebook.", parts[0]);
    else snprintf(pre, sizeof pre, "%s.vq.layers.%d._codebook.", parts[1], k - 1);
    snprintf(nm, sizeof nm, "%sembedding_sum", pre);
    const float* sum = cget(t, n, nm, (int64_t)bins * RVQ_DIM, &ok);
    snprintf(nm, sizeof nm, "%scluster_usage", pre);
    const float* use = cget(t, n, nm, bins, &ok);
    if (!ok) break;
    /* Codebook::new (stt/model.rs:146-157): embedding = embedding_sum / max(usage, 1e-5),
     * half_norms = sum(embedding^2) / 2. */
    for (int j = 0; j < bins; j++) {
      float u = use[j] > 1e-5f ? use[j] : 1e-5f;
      float h = 0.0f;
      for (int d = 0; d < RVQ_DIM; d++) {
        float e = sum[(size_t)j * RVQ_DIM + d] / u;
        q->emb[((size_t)k * bins + j) * RVQ_DIM + d] = e;
        h = h + e * e;
      }
      q->hn[(size_t)k * bins + j] = h * 0.5f;
    }
  }
  if (!ok) {
    orc_rvq_free(q);
    return NULL;
  }
  return q;
}

void orc_rvq_free(orc_rvq* q) {
  if (!q) return;
  free(q->proj[0]);
  free(q->proj[1]);
  free(q->emb);
  free(q->hn);
  free(q);
}

int orc_rvq_distances(orc_rvq* q, int k, const float* r, float* dist) {
  for (int j = 0; j < q->bins; j++) {
    const float* e = q->emb + ((size_t)k * q->bins + j) * RVQ_DIM;
    float acc = 0.0f;
    for (int d = 0; d < RVQ_DIM; d++) acc = fmaf(e[d], r[d], acc);
    dist[j] = q->hn[(size_t)k * q->bins + j] - acc; /* half_norms - dot (Codebook::encode) */
  }
  return 0;
}

/* Quantizer::encode: the first codebook on rvq_first's projection, the others residually on
 * rvq_rest's; argmin keeps the first minimum. */
int orc_rvq_encode(orc_rvq* q, const float* latent, int frames, uint32_t* codes) {
  float res[RVQ_DIM], x[RVQ_IN];
  float* dist = (float*)malloc(sizeof(float) * (size_t)q->bins);
  for (int f = 0; f < frames; f++) {
    for (int c = 0; c < RVQ_IN; c++) x[c] = latent[(size_t)c * frames + f];
    for (int k = 0; k < q->n_q; k++) {
      if (k <= 1) {
        const float* w = q->proj[k];
        for (int d = 0; d < RVQ_DIM; d++) {
          float acc = 0.0f;
          for (int c = 0; c < RVQ_IN; c++) acc = fmaf(w[(size_t)d * RVQ_IN + c], x[c], acc);
          res[d] = acc;
        }
      }
      orc_rvq_distances(q, k, res, dist);
      int best = 0;
      for (int j = 1; j < q->bins; j++)
        if (dist[j] < dist[best]) best = j;
      codes[(size_t)f * q->n_q + k] = (uint32_t)best;
      const float* e = q->emb + ((size_t)k * q->bins + best) * RVQ_DIM;
      for (int d = 0; d < RVQ_DIM; d++) res[d] = res[d] - e[d];
    }
  }
  free(dist);
  return 0;
}
