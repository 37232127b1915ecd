// Continuous-batching decoder: many independent sessions share one paged KV
// pool and one set of weights; every decode step packs the active sessions'
// next tokens into one batch (ragged KV lengths, per-session page tables).
//
// The reference decodes one session per AsrTextDecoder with a contiguous
// [max_seq, 8, 128] cache (src/model/asr_text_decoder.cu:309-318) and one
// pipeline thread per session (src/pipeline/asr_worker.cc:270-416); this is
// the batched replacement: projections run on the tcgen05 GEMM with M = 128
// weight rows x N = batch tokens, attention is flash-decoding over each row's
// own page table, and joins / leaves only edit host-side page lists and the
// device page table.
#include <algorithm>
#include <cstring>
#include <map>
#include <set>

#include "common.cuh"
#include "engine.h"

namespace orx {

namespace {
constexpr int kSplitPages = 32;  // pages per attention split (4 double-buffered groups)
constexpr int kPartFloats = 2 * 132;

// tokens[r] = next_tok[row_table[r]]; x[r] = embed[tokens[r]] (fp32).
__global__ void gather_tokens_embed(const int* next_tok, const int* row_table, const uint16_t* embed,
                                    int* tokens, float* x) {
  pdl_wait();
  const int r = blockIdx.x;
  const int tok = next_tok[row_table[r]];
  if (threadIdx.x == 0) tokens[r] = tok;
  const uint16_t* src = embed + (long long)tok * kHidden;
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) x[(long long)r * kHidden + i] = bf2f(src[i]);
}

// Row-wise argmax of logits [rows, n], split over kArgmaxChunks CTAs per row
// (grid (chunks, rows)): each CTA folds its slice into a 64-bit key
// (orderable value << 32 | ~index, so equal values resolve to the lowest
// index) with atomicMax on keys[r]; the last CTA of the row (ticket on
// cnt[r]) writes next_tok[row_table[r]] and out[r] and resets keys[r] and
// cnt[r] for the next launch. Session sid = row_table[r] excludes ids
// ban[sid].x and .y while ban[sid].z > 0, and each argmax of the session
// counts ban[sid].z down by one (the ban window of DecodeGreedy,
// src/model/asr_text_decoder.cu:698-857: the argmax producing token k bans
// the EOS ids iff k < ban_steps).
constexpr int kArgmaxChunks = 16;

__global__ void __launch_bounds__(512) rows_argmax(const float* logits, int n, const int* row_table,
                                                   int* next_tok, int* out, int4* ban,
                                                   unsigned long long* keys, int* cnt) {
  pdl_wait();
  __shared__ unsigned long long sb[16];
  const int r = blockIdx.y;
  const float* x = logits + (long long)r * n;
  const int sid = row_table[r];
  const int4 bn = ban[sid];
  const int b0 = bn.z > 0 ? bn.x : -1, b1 = bn.z > 0 ? bn.y : -1;
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int i0 = blockIdx.x * per, i1 = i0 + per < n ? i0 + per : n;
  unsigned long long best = 0ull;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = x[i];
    if (v != v || i == b0 || i == b1) continue;
    const unsigned long long k = argmax_key(v, i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) b = sb[w] > b ? sb[w] : b;
    if (b) atomicMax(keys + r, b);
    __threadfence();
    if (atomicAdd(cnt + r, 1) == static_cast<int>(gridDim.x) - 1) {
      __threadfence();
      const unsigned long long k = atomicExch(keys + r, 0ull);
      const int tok = k ? argmax_key_index(k) : 0;
      next_tok[sid] = tok;
      if (out) out[r] = tok;
      if (bn.z > 0) ban[sid].z = bn.z - 1;
      cnt[r] = 0;
    }
  }
}

// x_last[i] = x[last_row[i]]
__global__ void gather_rows(const float* x, const int* rows, float* out) {
  pdl_wait();
  const int i = blockIdx.x;
  const float* src = x + (long long)rows[i] * kHidden;
  for (int j = threadIdx.x; j < kHidden; j += blockDim.x) out[(long long)i * kHidden + j] = src[j];
}
}  // namespace

BatchDecoder::BatchDecoder(Model* m, int max_sessions, int max_batch, int pool_pages,
                           int max_pages_per_session)
    : model(m), max_sessions_(max_sessions), max_batch_(max_batch), mps_(max_pages_per_session) {
  if (max_sessions <= 0 || max_batch <= 0 || pool_pages <= 0 || max_pages_per_session <= 0)
    throw std::invalid_argument("invalid batch decoder sizes");
  if ((long long)max_pages_per_session * kPage > m->rope_positions)
    throw std::invalid_argument("max_pages_per_session exceeds the model's max_seq_len");
  kv_ = new KvPool(m->cfg.num_layers, pool_pages);
  free_pages_.resize(pool_pages);
  for (int i = 0; i < pool_pages; ++i) free_pages_[i] = pool_pages - 1 - i;
  sessions_.resize(max_sessions);
  h_table_.assign((size_t)max_sessions * mps_, 0);
  d_table_ = dalloc<int>((size_t)max_sessions * mps_);
  ORX_CHECK(cudaMemset(d_table_, 0, sizeof(int) * (size_t)max_sessions * mps_));
  d_next_tok_ = dalloc<int>(max_sessions);
  d_ban_ = dalloc<int4>(max_sessions);
  ORX_CHECK(cudaMemset(d_ban_, 0, sizeof(int4) * max_sessions));
  {  // argmax scratch, one key and one ticket per row; reset by its last CTA
    const int rows = std::max(max_sessions, max_batch);
    d_amax_keys_ = dalloc<unsigned long long>(rows);
    d_amax_cnt_ = dalloc<int>(rows);
    ORX_CHECK(cudaMemset(d_amax_keys_, 0, sizeof(unsigned long long) * rows));
    ORX_CHECK(cudaMemset(d_amax_cnt_, 0, sizeof(int) * rows));
  }
  ORX_CHECK(cudaMemset(d_next_tok_, 0, sizeof(int) * max_sessions));
  st_ = dalloc<StepState>(1);
  StepState init = {};
  ORX_CHECK(cudaMemcpy(st_, &init, sizeof(init), cudaMemcpyHostToDevice));
  ORX_CHECK(cudaMallocHost(&h_rows_, sizeof(int) * 2 * 65536));
  for (int b = 0; b < 2; ++b) {
    ORX_CHECK(cudaMallocHost(&h_step_[b], sizeof(int) * 2 * max_batch));
    ORX_CHECK(cudaMallocHost(&h_tbl_[b], sizeof(int) * h_table_.size()));
    ORX_CHECK(cudaEventCreateWithFlags(&ev_rows_[b], cudaEventDisableTiming));
    ORX_CHECK(cudaEventCreateWithFlags(&ev_table_[b], cudaEventDisableTiming));
  }
  ORX_CHECK(cudaMallocHost(&h_out_, sizeof(int) * max_batch));
  // Step buffers and the step workspace, sized once for every batch size up
  // to max_batch: the four layer projections and the lm_head.
  alloc_rows(stepb_, max_batch);
  ensure_logits(stepb_, max_batch);
  size_t need = 0;
  const int sms = m->num_sms;
  for (int n = 1; n <= max_batch; ++n)
    for (size_t f : {proj_ws_floats(kQkvDim, kHidden, n, sms), proj_ws_floats(kHidden, kQDim, n, sms),
                     proj_ws_floats(2 * kInter, kHidden, n, sms), proj_ws_floats(kHidden, kInter, n, sms),
                     proj_ws_floats(m->cfg.vocab_size, kHidden, n, sms)})
      need = std::max(need, f);
  step_ws_.reserve(need, nullptr);
}

BatchDecoder::~BatchDecoder() {
  delete kv_;
  graphs_.clear();
  stepb_.release();
  preb_.release();
  for (void* p : {(void*)d_table_, (void*)d_next_tok_, (void*)d_ban_, (void*)d_amax_keys_,
                  (void*)d_amax_cnt_, (void*)st_, (void*)d_tiles_})
    if (p) cudaFree(p);
  if (h_rows_) cudaFreeHost(h_rows_);
  if (h_tiles_) cudaFreeHost(h_tiles_);
  for (int b = 0; b < 2; ++b) {
    if (h_step_[b]) cudaFreeHost(h_step_[b]);
    if (h_tbl_[b]) cudaFreeHost(h_tbl_[b]);
    if (ev_rows_[b]) cudaEventDestroy(ev_rows_[b]);
    if (ev_table_[b]) cudaEventDestroy(ev_table_[b]);
  }
  if (h_out_) cudaFreeHost(h_out_);
}

void BatchDecoder::RowBufs::release() {
  for (void* p : {(void*)x, (void*)xn, (void*)qkv, (void*)attn, (void*)act, (void*)part,
                  (void*)counters, (void*)rows, (void*)tokens, (void*)out, (void*)logits})
    if (p) cudaFree(p);
  *this = RowBufs{};
}

// (Re)allocates `b` for at least `rows` rows; the caller has made sure that no
// queued work still uses the old buffers.
void BatchDecoder::alloc_rows(RowBufs& b, int rows) {
  if (rows <= b.cap) return;
  if (b.cap > 0) ORX_CHECK(cudaDeviceSynchronize());
  const int cap = std::max(rows, 64);
  float* lg = b.logits;
  const int lcap = b.logits_cap;
  b.logits = nullptr;
  b.release();
  b.logits = lg;
  b.logits_cap = lcap;
  b.x = dalloc<float>((size_t)cap * kHidden);
  b.xn = dalloc<uint16_t>((size_t)cap * kHidden);
  b.qkv = dalloc<float>((size_t)cap * kQkvDim);
  b.attn = dalloc<uint16_t>((size_t)cap * kQDim);
  b.act = dalloc<uint16_t>((size_t)cap * kInter);
  const int nsplit_cap = (mps_ + kSplitPages - 1) / kSplitPages;
  b.part = dalloc<float>((size_t)cap * kKvHeads * nsplit_cap * kPartFloats);
  b.counters = dalloc<int>((size_t)cap * kKvHeads);
  ORX_CHECK(cudaMemset(b.counters, 0, sizeof(int) * (size_t)cap * kKvHeads));
  b.rows = dalloc<int>((size_t)cap * 4);
  b.tokens = dalloc<int>(cap);
  b.out = dalloc<int>(cap);
  b.cap = cap;
  if (&b == &stepb_) ++step_realloc_;
}

void BatchDecoder::ensure_logits(RowBufs& b, int rows) {
  if (rows <= b.logits_cap) return;
  if (b.logits) {
    ORX_CHECK(cudaDeviceSynchronize());
    cudaFree(b.logits);
  }
  b.logits = dalloc<float>((size_t)rows * model->cfg.vocab_size);
  b.logits_cap = rows;
  if (&b == &stepb_) ++step_realloc_;
}

int BatchDecoder::create_session() {
  for (int i = 0; i < max_sessions_; ++i)
    if (!sessions_[i].live) {
      sessions_[i] = Session{};
      sessions_[i].live = true;
      return i;
    }
  return -1;
}

void BatchDecoder::check_sid(int sid) const {
  if (sid < 0 || sid >= max_sessions_ || !sessions_[sid].live)
    throw std::invalid_argument("unknown session id");
}

void BatchDecoder::free_session(int sid) {
  check_sid(sid);
  for (int p : sessions_[sid].pages) free_pages_.push_back(p);
  sessions_[sid] = Session{};
  const int4 none = {-1, -1, 0, 0};
  ORX_CHECK(cudaMemcpy(d_ban_ + sid, &none, sizeof(none), cudaMemcpyHostToDevice));
}

void BatchDecoder::next_tokens(const int* sids, int n, int* out, cudaStream_t s) const {
  for (int i = 0; i < n; ++i) check_sid(sids[i]);
  std::vector<int> all(max_sessions_);
  ORX_CHECK(cudaStreamSynchronize(s));
  ORX_CHECK(cudaMemcpy(all.data(), d_next_tok_, sizeof(int) * max_sessions_, cudaMemcpyDeviceToHost));
  for (int i = 0; i < n; ++i) out[i] = all[sids[i]];
}

void BatchDecoder::set_ban(int sid, int ban0, int ban1, int steps, cudaStream_t s) {
  check_sid(sid);
  if (steps < 0) throw std::invalid_argument("negative ban window");
  const int4 v = {ban0, ban1, steps, 0};
  // pageable source: the copy has consumed `v` when the call returns
  ORX_CHECK(cudaMemcpyAsync(d_ban_ + sid, &v, sizeof(v), cudaMemcpyHostToDevice, s));
}

int BatchDecoder::cache_len(int sid) const {
  check_sid(sid);
  return sessions_[sid].len;
}

void BatchDecoder::truncate(int sid, int len) {
  check_sid(sid);
  Session& s = sessions_[sid];
  if (len < 0 || len > s.len) throw std::invalid_argument("bad truncate length");
  s.len = len;
  const int keep = (len + kPage - 1) / kPage;
  while ((int)s.pages.size() > keep) {
    free_pages_.push_back(s.pages.back());
    s.pages.pop_back();
  }
}

// Makes session `sid` own pages for positions [0, new_len); false when the
// pool or the session's page table is exhausted (nothing is allocated then).
bool BatchDecoder::reserve(int sid, int new_len) {
  Session& s = sessions_[sid];
  const int need = (new_len + kPage - 1) / kPage;
  if (need > mps_) return false;
  const int extra = need - static_cast<int>(s.pages.size());
  if (extra <= 0) return true;
  if (extra > static_cast<int>(free_pages_.size())) return false;
  for (int i = 0; i < extra; ++i) {
    const int p = free_pages_.back();
    free_pages_.pop_back();
    h_table_[(size_t)sid * mps_ + s.pages.size()] = p;
    s.pages.push_back(p);
  }
  dirty_ = true;
  return true;
}

// Whether every session can grow by lens[i] rows (no allocation happens).
bool BatchDecoder::fits(const int* sids, const int* lens, int n) const {
  long long extra = 0;
  for (int i = 0; i < n; ++i) {
    const Session& s = sessions_[sids[i]];
    const int need = (s.len + lens[i] + kPage - 1) / kPage;
    if (need > mps_) return false;
    extra += std::max(0, need - static_cast<int>(s.pages.size()));
  }
  return extra <= static_cast<long long>(free_pages_.size());
}

void BatchDecoder::upload_table(cudaStream_t st) {
  if (!dirty_) return;
  const int b = table_count_++ & 1;
  ORX_CHECK(cudaEventSynchronize(ev_table_[b]));  // that staging copy has been consumed
  std::memcpy(h_tbl_[b], h_table_.data(), sizeof(int) * h_table_.size());
  ORX_CHECK(cudaMemcpyAsync(d_table_, h_tbl_[b], sizeof(int) * h_table_.size(),
                            cudaMemcpyHostToDevice, st));
  ORX_CHECK(cudaEventRecord(ev_table_[b], st));
  dirty_ = false;
}

// Shared per-layer body over `rows` rows of b.x whose (session, position) are in
// b.rows = [row_table | row_pos]. fused: decode mode (q/k norm, RoPE and the
// K/V store inside attention); otherwise the prefill store kernel runs first.
void BatchDecoder::layers(RowBufs& b, GemmWs& ws, int rows, int max_len, bool fused,
                          cudaStream_t s) {
  const auto& c = model->cfg;
  const int* row_table = b.rows;
  const int* row_pos = b.rows + b.cap;
  const int sms = model->num_sms;
  const int nsplit = ((max_len + kPage - 1) / kPage + kSplitPages - 1) / kSplitPages;
  int* err = &st_->err;
  for (int l = 0; l < c.num_layers; ++l) {
    const Model::Layer& L = model->layers[l];
    uint16_t* kvl = kv_->layer(l);
    // later layers' input norm comes fused with the previous down projection
    if (l == 0) launch_rmsnorm_bf16(b.x, L.in_ln, b.xn, rows, c.rms_norm_eps, s);
    run_proj(ws, b.xn, L.qkv, kQkvDim, kHidden, rows, kEpiStore, b.qkv, nullptr, kQkvDim, err, sms, s);
    if (!fused)
      launch_qk_norm_rope_store(b.qkv, rows, L.q_norm, L.k_norm, model->rope_cos, model->rope_sin,
                                kvl, d_table_, mps_, row_table, row_pos, 0, s);
    if (fused) {
      AttnArgs a = {};
      a.qkv = b.qkv;
      a.qkv_stride = kQkvDim;
      a.q_norm_w = L.q_norm;
      a.k_norm_w = L.k_norm;
      a.rope_cos = model->rope_cos;
      a.rope_sin = model->rope_sin;
      a.kv_layer = kvl;
      a.page_table = d_table_;
      a.max_pages = mps_;
      a.row_table = row_table;
      a.row_pos = row_pos;
      a.rows = rows;
      a.fused_kv = fused ? 1 : 0;
      a.nsplit_max = nsplit;
      a.pages_per_split = kSplitPages;
      a.part = b.part;
      a.counters = b.counters;
      a.out = b.attn;
      a.err = err;
      a.kv_row0 = l * kv_->pages * 2 * kKvHeads * kPage;
      launch_attention(a, kv_->base, (long long)kv_->num_layers * kv_->pages * 2 * kKvHeads * kPage, s);
    } else {
      PrefillAttnArgs pa = {};
      pa.qkv = b.qkv;
      pa.qkv_stride = kQkvDim;
      pa.tiles = d_tiles_;
      pa.page_table = d_table_;
      pa.max_pages = mps_;
      pa.kv_row0 = l * kv_->pages * 2 * kKvHeads * kPage;
      pa.out = b.attn;
      pa.err = err;
      launch_attn_prefill(pa, ntiles_, kv_->base,
                          (long long)kv_->num_layers * kv_->pages * 2 * kKvHeads * kPage, s);
    }
    run_proj(ws, b.attn, L.o, kHidden, kQDim, rows, kEpiResid, b.x, nullptr, kHidden, err, sms, s,
             L.post_ln, b.xn, c.rms_norm_eps);
    run_proj(ws, b.xn, L.gateup, 2 * kInter, kHidden, rows, kEpiSwiglu, nullptr, b.act, kInter, err, sms, s);
    // the next layer's input norm, or in a decode step the final norm
    const float* next_norm = l + 1 < c.num_layers ? model->layers[l + 1].in_ln
                                                   : (fused ? model->final_norm : nullptr);
    run_proj(ws, b.act, L.down, kHidden, kInter, rows, kEpiResid, b.x, nullptr, kHidden, err, sms, s,
             next_norm, b.xn, c.rms_norm_eps);
  }
}

void BatchDecoder::prefill(const int* sids, const int* lens, int n, const float* host_embeds,
                           cudaStream_t s) {
  if (n <= 0) return;
  int total = 0, max_len = 0;
  for (int i = 0; i < n; ++i) {
    check_sid(sids[i]);
    if (lens[i] <= 0) throw std::invalid_argument("empty prefill");
    for (int j = 0; j < i; ++j)
      if (sids[j] == sids[i]) throw std::invalid_argument("session listed twice");
    total += lens[i];
  }
  if (total > 65536 / 2) throw std::invalid_argument("too many prefill rows in one call");
  if (!fits(sids, lens, n)) throw std::invalid_argument("KV page pool exhausted");
  for (int i = 0; i < n; ++i) reserve(sids[i], sessions_[sids[i]].len + lens[i]);
  RowBufs& b = preb_;
  alloc_rows(b, std::max(total, n));
  ensure_logits(b, n);
  const int cap = b.cap;
  // rows: [row_table (cap) | row_pos (cap)], then the last-row list
  int r = 0;
  std::vector<int> last(n);
  for (int i = 0; i < n; ++i) {
    const Session& ss = sessions_[sids[i]];
    for (int t = 0; t < lens[i]; ++t, ++r) {
      h_rows_[r] = sids[i];
      h_rows_[cap + r] = ss.len + t;
    }
    last[i] = r - 1;
    max_len = std::max(max_len, ss.len + lens[i]);
  }
  // attention tiles: runs of consecutive rows of one session
  {
    const int tr = prefill_tile_rows();
    std::vector<PrefillTile> tiles;
    int row = 0;
    for (int i = 0; i < n; ++i) {
      const int base = sessions_[sids[i]].len;
      for (int t0 = 0; t0 < lens[i]; t0 += tr)
        tiles.push_back({sids[i], base + t0, std::min(tr, lens[i] - t0), row + t0});
      row += lens[i];
    }
    // longest key range first: the launch's first wave takes the heaviest
    // (tile, head) items and the short ones fill in behind them
    std::stable_sort(tiles.begin(), tiles.end(), [](const PrefillTile& x, const PrefillTile& y) {
      return x.pos0 + x.nrows > y.pos0 + y.nrows;
    });
    ntiles_ = static_cast<int>(tiles.size());
    if (ntiles_ > tiles_cap_) {
      if (d_tiles_) cudaFree(d_tiles_);
      if (h_tiles_) cudaFreeHost(h_tiles_);
      d_tiles_ = dalloc<PrefillTile>(ntiles_);
      ORX_CHECK(cudaMallocHost(&h_tiles_, sizeof(PrefillTile) * ntiles_));
      tiles_cap_ = ntiles_;
    }
    std::memcpy(h_tiles_, tiles.data(), sizeof(PrefillTile) * ntiles_);
    ORX_CHECK(cudaMemcpyAsync(d_tiles_, h_tiles_, sizeof(PrefillTile) * ntiles_,
                              cudaMemcpyHostToDevice, s));
  }
  upload_table(s);
  ORX_CHECK(cudaMemcpyAsync(b.rows, h_rows_, sizeof(int) * 2 * cap, cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaMemcpyAsync(b.x, host_embeds, sizeof(float) * (size_t)total * kHidden,
                            cudaMemcpyHostToDevice, s));
  layers(b, pre_ws_, total, max_len, false, s);
  // final norm + lm_head on each session's last row -> first decoded token
  std::memcpy(h_rows_ + 2 * cap, last.data(), sizeof(int) * n);
  for (int i = 0; i < n; ++i) h_rows_[2 * cap + n + i] = sids[i];
  ORX_CHECK(cudaMemcpyAsync(b.tokens, h_rows_ + 2 * cap, sizeof(int) * n,
                            cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaMemcpyAsync(b.out, h_rows_ + 2 * cap + n, sizeof(int) * n,
                            cudaMemcpyHostToDevice, s));
  launch_pdl(gather_rows, dim3(n), dim3(256), 0, s, (const float*)b.x, (const int*)b.tokens,
             (float*)b.qkv);
  const auto& c = model->cfg;
  launch_rmsnorm_bf16(b.qkv, model->final_norm, b.xn, n, c.rms_norm_eps, s);
  run_proj(pre_ws_, b.xn, model->embed, c.vocab_size, kHidden, n, kEpiStore, b.logits, nullptr,
           c.vocab_size, &st_->err, model->num_sms, s);
  launch_pdl(rows_argmax, dim3(kArgmaxChunks, n), dim3(512), 0, s, (const float*)b.logits,
             c.vocab_size, (const int*)b.out, d_next_tok_, (int*)nullptr, d_ban_, d_amax_keys_,
             d_amax_cnt_);
  ORX_CHECK(cudaGetLastError());
  ORX_CHECK(cudaStreamSynchronize(s));  // h_rows_ is reused by the next call
  for (int i = 0; i < n; ++i) sessions_[sids[i]].len += lens[i];
}

// Kernels of one decode step for n rows whose (session, position) are in
// stepb_.rows; every varying input lives in device memory, so the sequence is
// captured once per batch size and replayed as a CUDA graph.
void BatchDecoder::record_step(int n, cudaStream_t s) {
  RowBufs& b = stepb_;
  launch_pdl(gather_tokens_embed, dim3(n), dim3(256), 0, s, (const int*)d_next_tok_,
             (const int*)b.rows, (const uint16_t*)model->embed, b.tokens, b.x);
  layers(b, step_ws_, n, mps_ * kPage, true, s);  // ends with the final norm of every row in b.xn
  const auto& c = model->cfg;
  run_proj(step_ws_, b.xn, model->embed, c.vocab_size, kHidden, n, kEpiStore, b.logits, nullptr,
           c.vocab_size, &st_->err, model->num_sms, s);
  launch_pdl(rows_argmax, dim3(kArgmaxChunks, n), dim3(512), 0, s, (const float*)b.logits,
             c.vocab_size, (const int*)b.rows, d_next_tok_, b.out, d_ban_, d_amax_keys_,
             d_amax_cnt_);
}

void BatchDecoder::step(const int* sids, int n, int* host_tokens_out, cudaStream_t s) {
  if (n <= 0) return;
  if (n > max_batch_) throw std::invalid_argument("batch larger than max_batch");
  for (int i = 0; i < n; ++i) {
    check_sid(sids[i]);
    if (sessions_[sids[i]].len <= 0) throw std::invalid_argument("session has no prefix");
    for (int j = 0; j < i; ++j)
      if (sids[j] == sids[i]) throw std::invalid_argument("session listed twice");
  }
  {
    std::vector<int> ones(n, 1);
    if (!fits(sids, ones.data(), n)) throw std::invalid_argument("KV page pool exhausted");
  }
  for (int i = 0; i < n; ++i) reserve(sids[i], sessions_[sids[i]].len + 1);
  upload_table(s);
  RowBufs& rb = stepb_;
  // double-buffered pinned staging: wait only for the copy issued two steps ago
  const int b = step_count_ & 1;
  ORX_CHECK(cudaEventSynchronize(ev_rows_[b]));
  int* stage = h_step_[b];
  for (int i = 0; i < n; ++i) {
    stage[i] = sids[i];
    stage[max_batch_ + i] = sessions_[sids[i]].len;
  }
  ORX_CHECK(cudaMemcpyAsync(rb.rows, stage, sizeof(int) * n, cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaMemcpyAsync(rb.rows + rb.cap, stage + max_batch_, sizeof(int) * n,
                            cudaMemcpyHostToDevice, s));
  ORX_CHECK(cudaEventRecord(ev_rows_[b], s));
  ++step_count_;

  // A graph is replayed only under the memory epoch it was captured in (the
  // step buffers are sized for max_batch up front, so the epoch stays put;
  // the check keeps any future reallocation from reaching a stale graph).
  const uint64_t epoch = step_epoch();
  cudaGraphExec_t g = graphs_.find(n, epoch);
  if (!g && !graphs_.warmed(n)) {
    record_step(n, s);  // eager first run
    graphs_.mark_warmed(n);
  } else {
    if (!g) {
      ORX_CHECK(cudaStreamSynchronize(s));
      cudaStream_t cs;
      ORX_CHECK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
      ORX_CHECK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
      record_step(n, cs);
      cudaGraph_t cg;
      ORX_CHECK(cudaStreamEndCapture(cs, &cg));
      ORX_CHECK(cudaGraphInstantiate(&g, cg, 0));
      ORX_CHECK(cudaGraphDestroy(cg));
      ORX_CHECK(cudaStreamDestroy(cs));
      if (step_epoch() != epoch)
        throw CudaError("step buffers were reallocated while a step graph was captured");
      graphs_.insert(n, epoch, g);
    }
    ORX_CHECK(cudaGraphLaunch(g, s));
  }
  ORX_CHECK(cudaGetLastError());
  for (int i = 0; i < n; ++i) sessions_[sids[i]].len += 1;
  if (host_tokens_out) {
    ORX_CHECK(cudaMemcpyAsync(h_out_, rb.out, sizeof(int) * n, cudaMemcpyDeviceToHost, s));
    ORX_CHECK(cudaStreamSynchronize(s));
    std::memcpy(host_tokens_out, h_out_, sizeof(int) * n);
  }
}

int BatchDecoder::device_error() const {
  int e = 0;
  ORX_CHECK(cudaMemcpy(&e, &st_->err, 4, cudaMemcpyDeviceToHost));
  return e;
}

}  // namespace orx
