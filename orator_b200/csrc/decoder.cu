// One-session decoder with the reference AsrTextDecoder semantics
// (src/model/asr_text_decoder.cu:338-899), rebuilt around paged KV, fused
// weight-streaming kernels and CUDA graphs of PDL-chained launches.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "engine.h"

namespace orx {

// Projection on the tcgen05 GEMM with split-K chosen so that about one wave
// of CTAs covers the SMs (the short projections o / down / qkv at small T).
GemmWs::~GemmWs() {
  if (ws) cudaFree(ws);
  if (cnt) cudaFree(cnt);
}

int proj_splits(int N, int K, int T, int num_sms) {
  // Split-K by a small cost model of the persistent GEMM, calibrated on B200
  // (64, 400 and 3200 token rows): rounds of items per CTA x k-blocks per item
  // x time per k-block, the largest of (a) the weight box at the CTA's share
  // of HBM bandwidth (about 55 GB/s per streaming CTA at most), (b) weight +
  // activation boxes at about 120 GB/s of L2-to-SM bandwidth, (c) the tensor
  // time of the tile; plus the reduction kernel, which reads and writes the
  // fp32 partials at about 3 TB/s and costs a launch.
  auto cost = [&](int sp) {
    const int bn = tc_token_tile(N, T, sp, num_sms);
    const int tiles = (N / 128) * ((T + bn - 1) / bn);
    const int items = tiles * sp, active = items < num_sms ? items : num_sms;
    const double rounds = (items + num_sms - 1) / num_sms;
    const double kb = K / 64.0 / sp;
    const double w_bytes = 128.0 * 64 * 2, x_bytes = bn * 64 * 2.0;
    const double per_sm_hbm = std::min(6.4e12 / active, 55e9);
    const double t_unit = std::max({w_bytes / per_sm_hbm, (w_bytes + x_bytes) / 120e9,
                                    2.0 * 128 * bn * 64 / 10.8e12});
    const double red = sp > 1 ? (sp * 8.0 * T * N) / 3e12 + 4e-6 : 0.0;
    return rounds * kb * t_unit + red;
  };
  int splits = 1;
  for (int sp = 2; sp <= 16; sp *= 2)
    if (K % (64 * sp) == 0 && K / sp >= 128 && cost(sp) < cost(splits)) splits = sp;
  return splits;
}

size_t proj_ws_floats(int N, int K, int T, int num_sms) {
  const int sp = proj_splits(N, K, T, num_sms);
  return sp > 1 ? (size_t)sp * T * N : 0;
}

void GemmWs::reserve(size_t floats, cudaStream_t s) {
  if (floats <= cap) return;
  ORX_CHECK(cudaStreamSynchronize(s));
  if (!cnt) {
    cnt = dalloc<int>(kTickets);
    ORX_CHECK(cudaMemset(cnt, 0, kTickets * sizeof(int)));
  }
  if (ws) cudaFree(ws);
  ws = dalloc<float>(floats);
  cap = floats;
  ++gen;
}

void run_proj(GemmWs& w, const uint16_t* X, const uint16_t* W, int N, int K, int T, int epi,
              float* out_f32, uint16_t* out_bf16, int ldo, int* err, int num_sms, cudaStream_t s,
              const float* norm_w, uint16_t* norm_out, float eps) {
  if (T <= 0) return;
  const int splits = proj_splits(N, K, T, num_sms);
  TcArgs g = {N, K, T, epi, out_f32, out_bf16, ldo, err, nullptr, norm_w, norm_out, eps};
  if (splits > 1) {
    w.reserve((size_t)splits * T * N, s);
    g.ws = w.ws;
  }
  launch_gemm_tc(X, W, g, splits, s);
}

namespace {
constexpr int kDecodePagesPerSplit = 8;  // flash-decoding split size at batch 1
constexpr int kPartStride = 2 * 132;
}  // namespace

Decoder::Decoder(Model* m, bool own) : model(m), own_model_(own) {
  const auto& c = model->cfg;
  max_pages_ = (c.max_seq_len + kPage - 1) / kPage;
  kv_ = new KvPool(c.num_layers, max_pages_);
  std::vector<int> ident(max_pages_);
  for (int i = 0; i < max_pages_; ++i) ident[i] = i;
  page_table_ = dalloc<int>(max_pages_);
  ORX_CHECK(cudaMemcpy(page_table_, ident.data(), max_pages_ * 4, cudaMemcpyHostToDevice));
  dx_ = dalloc<float>(kHidden);
  dqkv_ = dalloc<float>(kQkvDim);
  dattn_ = dalloc<uint16_t>(kQDim);
  dact_ = dalloc<uint16_t>(kInter);
  logits_ = dalloc<float>(c.vocab_size);
  ORX_CHECK(cudaMemset(logits_, 0, (size_t)c.vocab_size * 4));
  part_ = dalloc<float>((size_t)kKvHeads * ((max_pages_ + kDecodePagesPerSplit - 1) / kDecodePagesPerSplit) * kPartStride);
  counters_ = dalloc<int>(kKvHeads);
  ORX_CHECK(cudaMemset(counters_, 0, kKvHeads * 4));
  st_ = dalloc<StepState>(1);
  StepState init = {};
  ORX_CHECK(cudaMemcpy(st_, &init, sizeof(init), cudaMemcpyHostToDevice));
  d_tmp_tok_ = dalloc<int>(1);
  ORX_CHECK(cudaMallocHost(&h_tok_, sizeof(int)));
  // persistent decode kernel: usable when one CTA per SM fits and the context
  // stays within its attention split table
  const char* nomk = std::getenv("ORX_NO_MK");
  use_mk_ = !(nomk && nomk[0] == '1') && max_pages_ <= kMkMaxSplit * 8 &&
            c.num_layers <= kMkMaxLayers &&
            decode_mk_max_grid() > 0;
  cudaGetLastError();
  if (use_mk_) {
    std::vector<MkLayerW> lw(c.num_layers);
    for (int l = 0; l < c.num_layers; ++l) {
      const Model::Layer& L = model->layers[l];
      lw[l] = {L.qkv, L.o, L.gateup, L.down, L.in_ln, L.post_ln, L.q_norm, L.k_norm};
    }
    mk_layers_ = dalloc<MkLayerW>(c.num_layers);
    ORX_CHECK(cudaMemcpy(mk_layers_, lw.data(), sizeof(MkLayerW) * c.num_layers,
                         cudaMemcpyHostToDevice));
    mk_part_ = dalloc<float>((size_t)kKvHeads * kMkMaxSplit * kMkPart);
    mk_sync_ = dalloc<unsigned long long>(4);
  }
}

Decoder::~Decoder() {
  if (g1_) cudaGraphExecDestroy(g1_);
  if (gk_) cudaGraphExecDestroy(gk_);
  delete kv_;
  for (void* p : {(void*)page_table_, (void*)dx_, (void*)dqkv_, (void*)dattn_, (void*)dact_,
                  (void*)logits_, (void*)part_, (void*)counters_, (void*)st_, (void*)d_out_,
                  (void*)d_tmp_tok_, (void*)px_, (void*)pqkv_, (void*)pxn_, (void*)pattn_,
                  (void*)pact_, (void*)pcounters_, (void*)ppart_, (void*)d_tiles_, (void*)mk_layers_, (void*)mk_part_,
                  (void*)mk_sync_})
    if (p) cudaFree(p);
  if (h_out_) cudaFreeHost(h_out_);
  if (h_tok_) cudaFreeHost(h_tok_);
  if (h_stage_) cudaFreeHost(h_stage_);
  if (h_tiles_) cudaFreeHost(h_tiles_);
  if (own_model_) delete model;
}

void Decoder::truncate_cache(int len) {
  if (len < 0 || len > model->cfg.max_seq_len) throw std::invalid_argument("bad cache length");
  cache_len_ = len;
}

void Decoder::embed(int token, float* out) const {
  if (token < 0 || token >= model->cfg.vocab_size) throw std::invalid_argument("token id out of range");
  uint16_t row[kHidden];
  ORX_CHECK(cudaMemcpy(row, model->embed + (size_t)token * kHidden, sizeof(row),
                       cudaMemcpyDeviceToHost));
  for (int i = 0; i < kHidden; ++i) {
    const uint32_t u = static_cast<uint32_t>(row[i]) << 16;
    std::memcpy(out + i, &u, 4);
  }
}

int Decoder::device_error() const {
  int e = 0;
  ORX_CHECK(cudaMemcpy(&e, &st_->err, 4, cudaMemcpyDeviceToHost));
  return e;
}

void Decoder::ensure_prefill(int T) {
  if (T <= tcap_) return;
  int cap = std::max(T, 64);
  for (void* p : {(void*)px_, (void*)pqkv_, (void*)pxn_, (void*)pattn_, (void*)pact_,
                  (void*)pcounters_, (void*)ppart_})
    if (p) cudaFree(p);
  px_ = dalloc<float>((size_t)cap * kHidden);
  ppart_ = dalloc<float>((size_t)cap * kKvHeads *
                         ((max_pages_ + kDecodePagesPerSplit - 1) / kDecodePagesPerSplit) * kPartStride);
  pqkv_ = dalloc<float>((size_t)cap * kQkvDim);
  pxn_ = dalloc<uint16_t>((size_t)cap * kHidden);
  pattn_ = dalloc<uint16_t>((size_t)cap * kQDim);
  pact_ = dalloc<uint16_t>((size_t)cap * kInter);
  pcounters_ = dalloc<int>((size_t)cap * kKvHeads);
  ORX_CHECK(cudaMemset(pcounters_, 0, (size_t)cap * kKvHeads * 4));
  tcap_ = cap;
}

// Prefill forward (Forward, asr_text_decoder.cu:457-583) over T rows of px_.
void Decoder::forward_prefill(int T, int pos0, cudaStream_t s) {
  const auto& c = model->cfg;
  // attention tiles: consecutive rows of the single session
  const int tr = prefill_tile_rows();
  const int ntiles = (T + tr - 1) / tr;
  if (ntiles > tiles_cap_) {
    ORX_CHECK(cudaStreamSynchronize(s));
    if (d_tiles_) cudaFree(d_tiles_);
    if (h_tiles_) cudaFreeHost(h_tiles_);
    d_tiles_ = dalloc<PrefillTile>(ntiles);
    ORX_CHECK(cudaMallocHost(&h_tiles_, sizeof(PrefillTile) * ntiles));
    tiles_cap_ = ntiles;
  }
  ORX_CHECK(cudaStreamSynchronize(s));  // h_tiles_ may still feed an earlier copy
  for (int i = 0; i < ntiles; ++i) {  // longest key range first (see the batched prefill)
    const int k = ntiles - 1 - i;
    h_tiles_[i] = {0, pos0 + k * tr, std::min(tr, T - k * tr), k * tr};
  }
  ORX_CHECK(cudaMemcpyAsync(d_tiles_, h_tiles_, sizeof(PrefillTile) * ntiles,
                            cudaMemcpyHostToDevice, s));
  for (int l = 0; l < c.num_layers; ++l) {
    const Model::Layer& L = model->layers[l];
    uint16_t* kvl = kv_->layer(l);
    launch_rmsnorm_bf16(px_, L.in_ln, pxn_, T, c.rms_norm_eps, s);
    run_proj(gws_, pxn_, L.qkv, kQkvDim, kHidden, T, kEpiStore, pqkv_, nullptr, kQkvDim, &st_->err, model->num_sms, s);
    launch_qk_norm_rope_store(pqkv_, T, L.q_norm, L.k_norm, model->rope_cos, model->rope_sin,
                              kvl, page_table_, max_pages_, nullptr, nullptr, pos0, s);
    PrefillAttnArgs pa = {};
    pa.qkv = pqkv_;
    pa.qkv_stride = kQkvDim;
    pa.tiles = d_tiles_;
    pa.page_table = page_table_;
    pa.max_pages = max_pages_;
    pa.kv_row0 = l * kv_->pages * 2 * kKvHeads * kPage;
    pa.out = pattn_;
    pa.err = &st_->err;
    launch_attn_prefill(pa, ntiles, kv_->base,
                        (long long)kv_->num_layers * kv_->pages * 2 * kKvHeads * kPage, s);
    run_proj(gws_, pattn_, L.o, kHidden, kQDim, T, kEpiResid, px_, nullptr, kHidden, &st_->err, model->num_sms, s);
    launch_rmsnorm_bf16(px_, L.post_ln, pxn_, T, c.rms_norm_eps, s);
    run_proj(gws_, pxn_, L.gateup, 2 * kInter, kHidden, T, kEpiSwiglu, nullptr, pact_, kInter, &st_->err, model->num_sms, s);
    run_proj(gws_, pact_, L.down, kHidden, kInter, T, kEpiResid, px_, nullptr, kHidden, &st_->err, model->num_sms, s);
  }
  // Final norm of the last row + tied lm_head (+ argmax into the step state).
  GemvArgs g = {};
  g.W = model->embed;
  g.K = kHidden;
  g.units = c.vocab_size;
  g.act_mode = kActNorm;
  g.x = px_ + (size_t)(T - 1) * kHidden;
  g.norm_w = model->final_norm;
  g.eps = c.rms_norm_eps;
  g.epi = kEpiLogits;
  g.out_f32 = logits_;
  g.finalize = 0;
  g.st = st_;
  launch_gemv(g, model->num_sms, s);
  ORX_CHECK(cudaGetLastError());
}

void Decoder::prefill_at(const float* host_embeds, int T, int pos0, cudaStream_t s) {
  if (T <= 0) return;
  if (pos0 < 0 || pos0 + T > model->cfg.max_seq_len)
    throw std::invalid_argument("prefill exceeds max_seq_len");
  ensure_prefill(T);
  ORX_CHECK(cudaMemcpyAsync(px_, host_embeds, (size_t)T * kHidden * 4, cudaMemcpyHostToDevice, s));
  forward_prefill(T, pos0, s);
  cache_len_ = pos0 + T;
  ORX_CHECK(cudaStreamSynchronize(s));
}

void Decoder::prefill_at_device(const float* dev_embeds, int T, int pos0, cudaStream_t s) {
  if (T <= 0) return;
  if (pos0 < 0 || pos0 + T > model->cfg.max_seq_len)
    throw std::invalid_argument("prefill exceeds max_seq_len");
  ensure_prefill(T);
  ORX_CHECK(cudaMemcpyAsync(px_, dev_embeds, (size_t)T * kHidden * 4, cudaMemcpyDeviceToDevice, s));
  forward_prefill(T, pos0, s);
  cache_len_ = pos0 + T;
}

// One decode body: layer 0 gathers the embedding of *tok_ptr; the lm_head
// kernel leaves logits and the banned argmax in the step state.
void Decoder::record_body(cudaStream_t s, const int* tok_ptr, bool record, bool finalize,
                          int only) {
  const auto& c = model->cfg;
  const int sms = model->num_sms;
  auto on = [&](int k) { return only < 0 || only == k; };
  int tslot = 0;
  auto tr = [&]() { return trace_ ? trace_ + 4 * (tslot++) : nullptr; };
  for (int l = 0; l < (only < 0 ? c.num_layers : 1); ++l) {
    const Model::Layer& L = model->layers[l];
    GemvArgs q = {};
    q.W = L.qkv;
    q.K = kHidden;
    q.units = kQkvDim;
    q.norm_w = L.in_ln;
    q.eps = c.rms_norm_eps;
    if (l == 0 && only < 0) {
      q.act_mode = kActEmbedNorm;
      q.embed = model->embed;
      q.tok_ptr = tok_ptr;
      q.x_init = dx_;
      q.record = record ? 1 : 0;
    } else {
      q.act_mode = kActNorm;
      q.x = dx_;
    }
    q.epi = kEpiStore;
    q.out_f32 = dqkv_;
    q.st = st_;
    q.trace = tr();
    if (on(0)) launch_gemv(q, sms, s);

    AttnArgs a = {};
    a.qkv = dqkv_;
    a.qkv_stride = kQkvDim;
    a.q_norm_w = L.q_norm;
    a.k_norm_w = L.k_norm;
    a.rope_cos = model->rope_cos;
    a.rope_sin = model->rope_sin;
    a.kv_layer = kv_->layer(l);
    a.page_table = page_table_;
    a.max_pages = max_pages_;
    a.pos_scalar = &st_->pos;
    a.rows = 1;
    a.fused_kv = 1;
    a.nsplit_max = (max_pages_ + kDecodePagesPerSplit - 1) / kDecodePagesPerSplit;
    a.pages_per_split = kDecodePagesPerSplit;
    a.part = part_;
    a.counters = counters_;
    a.out = dattn_;
    a.err = &st_->err;
    a.trace = tr();
    a.kv_row0 = l * kv_->pages * 2 * kKvHeads * kPage;
    if (on(1)) launch_attention(a, kv_->base, (long long)kv_->num_layers * kv_->pages * 2 * kKvHeads * kPage, s);

    GemvArgs o = {};
    o.W = L.o;
    o.K = kQDim;
    o.units = kHidden;
    o.act_mode = kActBf16;
    o.act = dattn_;
    o.epi = kEpiResid;
    o.out_f32 = dx_;
    o.st = st_;
    o.trace = tr();
    if (on(2)) launch_gemv(o, sms, s);

    GemvArgs gu = {};
    gu.W = L.gateup;
    gu.K = kHidden;
    gu.units = kInter;
    gu.act_mode = kActNorm;
    gu.x = dx_;
    gu.norm_w = L.post_ln;
    gu.eps = c.rms_norm_eps;
    gu.epi = kEpiSwiglu;
    gu.out_bf16 = dact_;
    gu.st = st_;
    gu.trace = tr();
    if (on(3)) launch_gemv(gu, sms, s);

    GemvArgs d = {};
    d.W = L.down;
    d.K = kInter;
    d.units = kHidden;
    d.act_mode = kActBf16;
    d.act = dact_;
    d.epi = kEpiResid;
    d.out_f32 = dx_;
    d.st = st_;
    d.trace = tr();
    if (on(4)) launch_gemv(d, sms, s);
  }
  GemvArgs g = {};
  g.W = model->embed;
  g.K = kHidden;
  g.units = c.vocab_size;
  g.act_mode = kActNorm;
  g.x = dx_;
  g.norm_w = model->final_norm;
  g.eps = c.rms_norm_eps;
  g.epi = kEpiLogits;
  g.out_f32 = logits_;
  g.finalize = finalize ? 1 : 0;
  g.st = st_;
  g.trace = tr();
  if (on(5)) launch_gemv(g, sms, s);
}

// One cooperative launch decoding `steps` tokens from `pos0` (see decode_mk.cu).
void Decoder::launch_mk(const int* tok_ptr, int steps, int pos0, int count0, bool record,
                        bool finalize, int ban_steps, int ban0, int ban1, cudaStream_t s) {
  const auto& c = model->cfg;
  ORX_CHECK(cudaMemsetAsync(mk_sync_, 0, 4 * sizeof(unsigned long long), s));
  MkArgs a = {};
  a.layers = mk_layers_;
  a.L = c.num_layers;
  a.embed = model->embed;
  a.final_norm = model->final_norm;
  a.vocab = c.vocab_size;
  a.rope_cos = model->rope_cos;
  a.rope_sin = model->rope_sin;
  a.kv = kv_->base;
  a.kv_layer_stride = (long long)kv_->pages * kPageElems;
  a.page_table = page_table_;
  a.max_pages = max_pages_;
  a.st = st_;
  a.tok_ptr = tok_ptr;
  a.steps = steps;
  a.record = record ? 1 : 0;
  a.finalize = finalize ? 1 : 0;
  a.pos0 = pos0;
  a.count0 = count0;
  a.ban_steps = ban_steps;
  a.ban0 = ban0;
  a.ban1 = ban1;
  a.x = dx_;
  a.qkv = dqkv_;
  a.part = mk_part_;
  a.act_g = dact_;
  a.logits = logits_;
  a.best2 = mk_sync_;
  a.bar = reinterpret_cast<unsigned int*>(mk_sync_ + 2);
  a.eps = c.rms_norm_eps;
  a.trace = mk_trace_;
  a.trace_cta = mk_trace_cta_;
  ORX_CHECK(launch_decode_mk(a, model->num_sms, s));
}

void Decoder::decode_step_device(const int* d_token, int pos, cudaStream_t s) {
  if (pos < 0 || pos >= model->cfg.max_seq_len) throw std::invalid_argument("position out of range");
  cache_len_ = pos + 1;
  if (use_mk_) {
    launch_mk(d_token, 1, pos, 0, false, false, 0, -1, -1, s);
    return;
  }
  ORX_CHECK(cudaMemcpyAsync(&st_->pos, &pos, 4, cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaStreamSynchronize(s));  // `pos` is a stack value
  record_body(s, d_token, false, false);
  ORX_CHECK(cudaGetLastError());
}

void Decoder::decode_step(const float* host_embed, int pos, cudaStream_t s) {
  // The embedding row is uploaded and fed through the embed path by id only
  // when it is an exact table row; a general embedding runs as a 1-row prefill.
  if (pos < 0 || pos >= model->cfg.max_seq_len) throw std::invalid_argument("position out of range");
  prefill_at(host_embed, 1, pos, s);
}

int Decoder::argmax(int ban0, int ban1, cudaStream_t s) {
  launch_argmax(logits_, model->cfg.vocab_size, ban0, ban1, st_, d_tmp_tok_, s);
  ORX_CHECK(cudaMemcpyAsync(h_tok_, d_tmp_tok_, 4, cudaMemcpyDeviceToHost, s));
  ORX_CHECK(cudaStreamSynchronize(s));
  return *h_tok_;
}

void Decoder::argmax_to_device(int* d_out, int ban0, int ban1, cudaStream_t s) {
  launch_argmax(logits_, model->cfg.vocab_size, ban0, ban1, st_, d_out, s);
  ORX_CHECK(cudaGetLastError());
}

int Decoder::read_token_id(const int* d_token, cudaStream_t s) const {
  ORX_CHECK(cudaMemcpyAsync(h_tok_, d_token, 4, cudaMemcpyDeviceToHost, s));
  ORX_CHECK(cudaStreamSynchronize(s));
  return *h_tok_;
}

void Decoder::copy_logits(float* host_out, cudaStream_t s) const {
  ORX_CHECK(cudaStreamSynchronize(s));
  ORX_CHECK(cudaMemcpy(host_out, logits_, (size_t)model->cfg.vocab_size * 4,
                       cudaMemcpyDeviceToHost));
}

void Decoder::ensure_graphs(cudaStream_t s) {
  if (g1_) return;
  cudaStream_t cs;
  ORX_CHECK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  auto capture = [&](int steps) {
    ORX_CHECK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    for (int i = 0; i < steps; ++i) record_body(cs, &st_->tok, true, true);
    cudaGraph_t g;
    ORX_CHECK(cudaStreamEndCapture(cs, &g));
    cudaGraphExec_t e;
    ORX_CHECK(cudaGraphInstantiate(&e, g, 0));
    ORX_CHECK(cudaGraphDestroy(g));
    return e;
  };
  g1_ = capture(1);
  gk_ = capture(graph_steps);
  ORX_CHECK(cudaStreamDestroy(cs));
  (void)s;
}

// Greedy loop with the reference's control semantics (DecodeGreedy, eager
// path, asr_text_decoder.cu:698-857): seed argmax (banned iff ban_steps > 0),
// the argmax producing token k bans eos0/eos1 iff k < ban_steps, stop on EOS
// (excluded) or six equal tokens in a row, checked once per batch; the cache
// length counts every step that ran. Each step is on-device end to end.
std::vector<int> Decoder::decode_greedy(int start_pos, int max_new, int eos0, int eos1,
                                        int ban_steps, int batch, cudaStream_t s) {
  std::vector<int> out;
  if (max_new <= 0) return out;
  if (start_pos < 0 || start_pos + max_new > model->cfg.max_seq_len)
    throw std::invalid_argument("decode would exceed max_seq_len");
  if (batch < 1) batch = 1;
  if (out_cap_ < max_new) {
    if (d_out_) cudaFree(d_out_);
    if (h_out_) cudaFreeHost(h_out_);
    d_out_ = dalloc<int>(max_new);
    ORX_CHECK(cudaMallocHost(&h_out_, sizeof(int) * max_new));
    out_cap_ = max_new;
  }
  if (!use_mk_) ensure_graphs(s);
  ORX_CHECK(cudaStreamSynchronize(s));
  StepState init = {};
  init.pos = start_pos;
  init.count = 0;
  init.ban_steps = ban_steps;
  init.ban0 = eos0;
  init.ban1 = eos1;
  init.out_cap = out_cap_;
  init.out = d_out_;
  ORX_CHECK(cudaMemcpy(st_, &init, sizeof(init), cudaMemcpyHostToDevice));
  const bool seed_ban = ban_steps > 0;
  launch_argmax(logits_, model->cfg.vocab_size, seed_ban ? eos0 : -1, seed_ban ? eos1 : -1, st_,
                nullptr, s);
  ORX_CHECK(cudaGetLastError());

  auto harvest = [&](int upto) {
    for (int i = static_cast<int>(out.size()); i < upto; ++i) {
      const int t = h_out_[i];
      if (t == eos0 || t == eos1) return true;
      out.push_back(t);
      if (out.size() >= 6) {
        bool same = true;
        for (size_t k = out.size() - 6; k + 1 < out.size(); ++k)
          if (out[k] != out.back()) { same = false; break; }
        if (same) return true;
      }
    }
    return false;
  };
  int emitted = 0;
  while (emitted < max_new) {
    const bool next_ban = (emitted + 1) < ban_steps;
    const int this_batch = next_ban ? 1 : std::min(batch, max_new - emitted);
    int left = use_mk_ ? 0 : this_batch;
    if (use_mk_)
      launch_mk(&st_->tok, this_batch, start_pos + emitted, emitted, true, true, ban_steps, eos0,
                eos1, s);
    while (left >= graph_steps) {
      ORX_CHECK(cudaGraphLaunch(gk_, s));
      left -= graph_steps;
    }
    for (; left > 0; --left) ORX_CHECK(cudaGraphLaunch(g1_, s));
    ORX_CHECK(cudaMemcpyAsync(h_out_ + emitted, d_out_ + emitted, sizeof(int) * this_batch,
                              cudaMemcpyDeviceToHost, s));
    ORX_CHECK(cudaStreamSynchronize(s));
    emitted += this_batch;
    if (harvest(emitted)) break;
  }
  cache_len_ = start_pos + emitted;
  return out;
}

// Average device time per launch of each decode kernel class (qkv GEMV,
// attention, o GEMV, gate/up GEMV, down GEMV, lm_head GEMV), each launched
// `iters` times back to back between CUDA events on `s`. Diagnostic only: it
// overwrites the step buffers and the KV entry at the current position.
void Decoder::profile_kernels(int iters, float* ms, cudaStream_t s) {
  const int pos = cache_len_ > 0 ? cache_len_ - 1 : 0;
  ORX_CHECK(cudaMemcpyAsync(&st_->pos, &pos, 4, cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaStreamSynchronize(s));
  cudaEvent_t e0, e1;
  ORX_CHECK(cudaEventCreate(&e0));
  ORX_CHECK(cudaEventCreate(&e1));
  for (int k = 0; k < 6; ++k) {
    record_body(s, &st_->tok, false, false, k);  // warm-up
    ORX_CHECK(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; ++i) record_body(s, &st_->tok, false, false, k);
    ORX_CHECK(cudaEventRecord(e1, s));
    ORX_CHECK(cudaEventSynchronize(e1));
    float t = 0.f;
    ORX_CHECK(cudaEventElapsedTime(&t, e0, e1));
    ms[k] = t / iters;
  }
  ORX_CHECK(cudaEventDestroy(e0));
  ORX_CHECK(cudaEventDestroy(e1));
}

int Decoder::trace_ctas(int steps, unsigned long long* host_out, size_t out_len, cudaStream_t s) {
  if (!use_mk_) throw std::invalid_argument("the persistent decode kernel is not in use");
  const int per = 5 * model->cfg.num_layers + 1, G = model->num_sms;
  const size_t n = ((size_t)steps * per + 1) * G * 2;
  if (out_len < (size_t)steps * per * G * 2) throw std::invalid_argument("out_len too small");
  unsigned long long* buf = dalloc<unsigned long long>(n);
  ORX_CHECK(cudaMemset(buf, 0, n * 8));
  mk_trace_cta_ = buf;
  launch_mk(&st_->tok, steps, cache_len_, 0, false, true, 0, -1, -1, s);
  mk_trace_cta_ = nullptr;
  ORX_CHECK(cudaStreamSynchronize(s));
  // slot k + 1 of the device buffer holds phase k (barrier numbers start at 1)
  ORX_CHECK(cudaMemcpy(host_out, buf + (size_t)G * 2, (size_t)steps * per * G * 2 * 8,
                       cudaMemcpyDeviceToHost));
  cudaFree(buf);
  cache_len_ += steps;
  return G;
}

// Debug timeline of `steps` eager decode bodies from the current cache end:
// per launch {first CTA start, last CTA past griddepcontrol.wait, last CTA end}
// in global-timer ns, written to host_out[steps * launches_per_step * 3].
int Decoder::trace_decode(int steps, unsigned long long* host_out, cudaStream_t s) {
  const int per = 5 * model->cfg.num_layers + 1;
  if (use_mk_) {
    // persistent kernel: CTA 0's barrier arrive / depart times, 2 per barrier
    const size_t n = 2 * ((size_t)steps * per + 1);
    unsigned long long* buf = dalloc<unsigned long long>(n);
    ORX_CHECK(cudaMemset(buf, 0, n * 8));
    mk_trace_ = buf;
    launch_mk(&st_->tok, steps, cache_len_, 0, false, true, 0, -1, -1, s);
    mk_trace_ = nullptr;
    ORX_CHECK(cudaStreamSynchronize(s));
    std::vector<unsigned long long> h(n);
    ORX_CHECK(cudaMemcpy(h.data(), buf, n * 8, cudaMemcpyDeviceToHost));
    cudaFree(buf);
    for (size_t i = 0; i < (size_t)steps * per * 3; ++i) host_out[i] = 0;
    for (size_t k = 1; k <= (size_t)steps * per; ++k) {  // launch slot k-1: {prev depart, arrive, depart}
      host_out[(k - 1) * 3] = h[2 * (k - 1) + 1];
      host_out[(k - 1) * 3 + 1] = h[2 * k];
      host_out[(k - 1) * 3 + 2] = h[2 * k + 1];
    }
    cache_len_ += steps;
    return per;
  }
  const size_t n = (size_t)steps * per * 4;
  std::vector<unsigned long long> init(n, 0ull);
  for (size_t i = 0; i < n; i += 4) init[i] = ~0ull;
  unsigned long long* buf = dalloc<unsigned long long>(n);
  ORX_CHECK(cudaMemcpy(buf, init.data(), n * 8, cudaMemcpyHostToDevice));
  int pos = cache_len_;
  ORX_CHECK(cudaMemcpy(&st_->pos, &pos, 4, cudaMemcpyHostToDevice));
  for (int i = 0; i < steps; ++i) {
    trace_ = buf + (size_t)i * per * 4;
    record_body(s, &st_->tok, false, true);
  }
  trace_ = nullptr;
  ORX_CHECK(cudaStreamSynchronize(s));
  ORX_CHECK(cudaMemcpy(init.data(), buf, n * 8, cudaMemcpyDeviceToHost));
  cudaFree(buf);
  for (size_t i = 0, j = 0; i < n; i += 4, j += 3) {
    host_out[j] = init[i];
    host_out[j + 1] = init[i + 1];
    host_out[j + 2] = init[i + 2];
  }
  cache_len_ = pos + steps;
  return per;
}

}  // namespace orx
