// extern "C" entry points declared in include/orx.h.
#include <cstring>
#include <exception>
#include <mutex>
#include <new>
#include <string>

#include "../../include/orx.h"
#include "common.cuh"
#include "engine.h"
#include "safetensors.h"

struct orx_decoder {
  orx::Decoder* dec = nullptr;
  int device = 0;
};

struct orx_layer32 {
  orx::Layer32* l = nullptr;
  int device = 0;
  float* d_io = nullptr;  // staging for host calls: [cap rows in | cap rows out]
  int cap = 0;
};

struct orx_vad {
  orx::BatchVad* v = nullptr;
  int device = 0;
};

struct orx_tower {
  orx::AudioTower* t = nullptr;
  int device = 0;
};

struct orx_sf {
  orx::Sortformer* s = nullptr;
  int device = 0;
  float* stage = nullptr;  // host calls: device copies of the inputs and outputs
  size_t cap = 0;
  float* ensure(size_t floats) {
    if (floats > cap) {
      orx::check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
      if (stage) cudaFree(stage);
      stage = orx::dalloc<float>(floats);
      cap = floats;
    }
    return stage;
  }
};

struct orx_batch {
  orx::BatchDecoder* b = nullptr;
  int device = 0;
};

namespace {
thread_local std::string g_err;

template <typename F>
int guard(F&& f) {
  try {
    f();
    return ORX_OK;
  } catch (const orx::CudaError& e) {
    g_err = e.what();
    return ORX_ECUDA;
  } catch (const std::invalid_argument& e) {
    g_err = e.what();
    return ORX_EINVAL;
  } catch (const std::bad_alloc&) {
    g_err = "host allocation failed";
    return ORX_EINTERNAL;
  } catch (const std::exception& e) {
    g_err = e.what();
    return ORX_EINVAL;
  }
}

void need(const void* p, const char* what) {
  if (!p) throw std::invalid_argument(std::string("null argument: ") + what);
}

// Calls run on the device the decoder was created on.
struct DeviceScope {
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) orx::check(cudaSetDevice(dev), "cudaSetDevice");
    restore = prev != dev;
  }
  ~DeviceScope() {
    if (restore) cudaSetDevice(prev);
  }
  int prev = 0;
  bool restore = false;
};

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

namespace orx {
void set_last_error(const char* msg) { g_err = msg; }
}  // namespace orx

extern "C" {

const char* orx_last_error(void) { return g_err.c_str(); }
int orx_version(void) { return 1; }

void orx_config_default(orx_config* c) {
  if (!c) return;
  c->hidden_size = 2048;
  c->num_layers = 28;
  c->num_q_heads = 16;
  c->num_kv_heads = 8;
  c->head_dim = 128;
  c->intermediate_size = 6144;
  c->vocab_size = 151936;
  c->rms_norm_eps = 1e-6f;
  c->rope_theta = 1000000.0f;
  c->max_seq_len = 2048;
  c->profile = 0;
  c->cuda_graph_enabled = 1;
}

int orx_decoder_create(const orx_config* cfg, orx_decoder** out) {
  return guard([&] {
    need(cfg, "cfg");
    need(out, "out");
    *out = nullptr;
    if (cfg->hidden_size != orx::kHidden || cfg->num_q_heads != orx::kQHeads ||
        cfg->num_kv_heads != orx::kKvHeads || cfg->head_dim != orx::kHeadDim ||
        cfg->intermediate_size != orx::kInter)
      throw std::invalid_argument("only the Qwen3-ASR-1.7B head geometry is supported");
    if (cfg->rms_norm_eps != 1e-6f) throw std::invalid_argument("rms_norm_eps must be 1e-6");
    orx::ModelConfig mc;
    mc.num_layers = cfg->num_layers;
    mc.vocab_size = cfg->vocab_size;
    mc.max_seq_len = cfg->max_seq_len;
    mc.rms_norm_eps = cfg->rms_norm_eps;
    mc.rope_theta = cfg->rope_theta;
    auto* h = new orx_decoder;
    try {
      orx::check(cudaGetDevice(&h->device), "cudaGetDevice");
      auto* m = new orx::Model(mc);
      h->dec = new orx::Decoder(m, true);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_decoder_destroy(orx_decoder* d) {
  if (!d) return;
  DeviceScope ds(d->device);
  delete d->dec;
  delete d;
}

int orx_decoder_set_tensor(orx_decoder* d, const char* name, const void* data, int dtype,
                           size_t numel, int on_device) {
  return guard([&] {
    need(d, "decoder");
    need(name, "name");
    need(data, "data");
    DeviceScope ds(d->device);
    d->dec->model->set_tensor(name, data, dtype, numel, on_device != 0);
  });
}

int orx_decoder_load_safetensors(orx_decoder* d, const char* dir) {
  return guard([&] {
    need(d, "decoder");
    need(dir, "model_dir");
    DeviceScope ds(d->device);
    orx::ShardedCheckpoint ck(dir);
    for (const auto& kv : ck.tensors()) {
      const auto& t = kv.second;
      int dtype;
      size_t es;
      if (t.dtype == "BF16") { dtype = 1; es = 2; }
      else if (t.dtype == "F32") { dtype = 0; es = 4; }
      else throw std::invalid_argument("unsupported dtype " + t.dtype + " for " + kv.first);
      if (kv.first.rfind("thinker.model.", 0) != 0 && kv.first != "thinker.lm_head.weight")
        continue;  // audio tower and other parts of the checkpoint
      d->dec->model->set_tensor(kv.first, t.data, dtype, t.nbytes / es, false);
    }
    if (!d->dec->model->complete()) throw std::invalid_argument("checkpoint is missing tensors");
  });
}

int orx_decoder_init_synthetic(orx_decoder* d, int seed) {
  return guard([&] {
    need(d, "decoder");
    DeviceScope ds(d->device);
    d->dec->model->init_synthetic(seed, 0);
  });
}

int orx_decoder_weights_complete(const orx_decoder* d, int* complete) {
  return guard([&] {
    need(d, "decoder");
    need(complete, "complete");
    *complete = d->dec->model->complete() ? 1 : 0;
  });
}

int orx_decoder_reset_cache(orx_decoder* d) {
  return guard([&] { need(d, "decoder"); d->dec->reset_cache(); });
}
int orx_decoder_truncate_cache(orx_decoder* d, int len) {
  return guard([&] { need(d, "decoder"); d->dec->truncate_cache(len); });
}
int orx_decoder_cache_len(const orx_decoder* d, int* out) {
  return guard([&] { need(d, "decoder"); need(out, "out"); *out = d->dec->cache_len(); });
}
int orx_decoder_embed(const orx_decoder* d, int token_id, float* out) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    DeviceScope ds(d->device);
    d->dec->embed(token_id, out);
  });
}

int orx_decoder_prefill_at(orx_decoder* d, const float* embeds, int T, int pos0, void* stream) {
  return guard([&] {
    need(d, "decoder");
    if (T > 0) need(embeds, "embeds");
    DeviceScope ds(d->device);
    d->dec->prefill_at(embeds, T, pos0, S(stream));
  });
}
int orx_decoder_prefill_at_device(orx_decoder* d, const float* e, int T, int pos0, void* stream) {
  return guard([&] {
    need(d, "decoder");
    if (T > 0) need(e, "embeds");
    DeviceScope ds(d->device);
    d->dec->prefill_at_device(e, T, pos0, S(stream));
  });
}
int orx_decoder_decode_step(orx_decoder* d, const float* embed, int pos, void* stream) {
  return guard([&] {
    need(d, "decoder");
    need(embed, "embed");
    DeviceScope ds(d->device);
    d->dec->decode_step(embed, pos, S(stream));
  });
}
int orx_decoder_decode_step_device(orx_decoder* d, const int* tok, int pos, void* stream) {
  return guard([&] {
    need(d, "decoder");
    need(tok, "d_token");
    DeviceScope ds(d->device);
    d->dec->decode_step_device(tok, pos, S(stream));
  });
}
int orx_decoder_argmax(orx_decoder* d, int ban0, int ban1, void* stream, int* out) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    DeviceScope ds(d->device);
    *out = d->dec->argmax(ban0, ban1, S(stream));
  });
}
int orx_decoder_argmax_to_device(orx_decoder* d, int* d_out, int ban0, int ban1, void* stream) {
  return guard([&] {
    need(d, "decoder");
    need(d_out, "d_out");
    DeviceScope ds(d->device);
    d->dec->argmax_to_device(d_out, ban0, ban1, S(stream));
  });
}
int orx_decoder_read_token_id(const orx_decoder* d, const int* tok, void* stream, int* out) {
  return guard([&] {
    need(d, "decoder");
    need(tok, "d_token");
    need(out, "out");
    DeviceScope ds(d->device);
    *out = d->dec->read_token_id(tok, S(stream));
  });
}
int orx_decoder_decode_greedy(orx_decoder* d, int start_pos, int max_new, int eos0, int eos1,
                              int ban_steps, int batch, void* stream, int* out_tokens,
                              int* n_out) {
  return guard([&] {
    need(d, "decoder");
    need(n_out, "n_out");
    if (max_new > 0) need(out_tokens, "out_tokens");
    DeviceScope ds(d->device);
    auto v = d->dec->decode_greedy(start_pos, max_new, eos0, eos1, ban_steps, batch, S(stream));
    if (!v.empty()) std::memcpy(out_tokens, v.data(), v.size() * sizeof(int));
    *n_out = static_cast<int>(v.size());
  });
}
int orx_decoder_copy_logits(const orx_decoder* d, float* out) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    DeviceScope ds(d->device);
    d->dec->copy_logits(out, 0);
  });
}
int orx_decoder_logits_device(const orx_decoder* d, const float** out) {
  return guard([&] { need(d, "decoder"); need(out, "out"); *out = d->dec->logits_device(); });
}
int orx_decoder_device_error(const orx_decoder* d, int* out) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    DeviceScope ds(d->device);
    *out = d->dec->device_error();
  });
}

int orx_decoder_profile_kernels(orx_decoder* d, int iters, void* stream, float* ms) {
  return guard([&] {
    need(d, "decoder");
    need(ms, "ms");
    if (iters < 1) throw std::invalid_argument("iters must be >= 1");
    DeviceScope ds(d->device);
    d->dec->profile_kernels(iters, ms, S(stream));
  });
}

int orx_decoder_trace_decode(orx_decoder* d, int steps, void* stream,
                             unsigned long long* out, int* launches_per_step) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    if (steps < 1) throw std::invalid_argument("steps must be >= 1");
    DeviceScope ds(d->device);
    const int per = d->dec->trace_decode(steps, out, S(stream));
    if (launches_per_step) *launches_per_step = per;
  });
}

int orx_decoder_trace_ctas(orx_decoder* d, int steps, void* stream, unsigned long long* out,
                           size_t out_len, int* grid) {
  return guard([&] {
    need(d, "decoder");
    need(out, "out");
    if (steps < 1) throw std::invalid_argument("steps must be >= 1");
    DeviceScope ds(d->device);
    const int g = d->dec->trace_ctas(steps, out, out_len, S(stream));
    if (grid) *grid = g;
  });
}

int orx_batch_create(orx_decoder* weights, int max_sessions, int max_batch, int pool_pages,
                     int max_pages_per_session, orx_batch** out) {
  return guard([&] {
    need(weights, "weights decoder");
    need(out, "out");
    *out = nullptr;
    DeviceScope ds(weights->device);
    auto* h = new orx_batch;
    h->device = weights->device;
    try {
      h->b = new orx::BatchDecoder(weights->dec->model, max_sessions, max_batch, pool_pages,
                                   max_pages_per_session);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_batch_destroy(orx_batch* b) {
  if (!b) return;
  DeviceScope ds(b->device);
  delete b->b;
  delete b;
}

int orx_batch_session_create(orx_batch* b, int* sid) {
  return guard([&] {
    need(b, "batch");
    need(sid, "sid");
    *sid = b->b->create_session();
    if (*sid < 0) throw std::invalid_argument("no free session slot");
  });
}

int orx_batch_session_free(orx_batch* b, int sid) {
  return guard([&] { need(b, "batch"); b->b->free_session(sid); });
}

int orx_batch_cache_len(const orx_batch* b, int sid, int* out) {
  return guard([&] { need(b, "batch"); need(out, "out"); *out = b->b->cache_len(sid); });
}

int orx_batch_truncate(orx_batch* b, int sid, int len) {
  return guard([&] { need(b, "batch"); b->b->truncate(sid, len); });
}

int orx_batch_free_pages(const orx_batch* b, int* out) {
  return guard([&] { need(b, "batch"); need(out, "out"); *out = b->b->free_pages(); });
}

int orx_batch_prefill(orx_batch* b, const int* sids, const int* lens, int n,
                      const float* embeds, void* stream) {
  return guard([&] {
    need(b, "batch");
    if (n > 0) { need(sids, "sids"); need(lens, "lens"); need(embeds, "embeds"); }
    DeviceScope ds(b->device);
    b->b->prefill(sids, lens, n, embeds, S(stream));
  });
}

int orx_batch_step(orx_batch* b, const int* sids, int n, int* tokens_out, void* stream) {
  return guard([&] {
    need(b, "batch");
    if (n > 0) need(sids, "sids");
    DeviceScope ds(b->device);
    b->b->step(sids, n, tokens_out, S(stream));
  });
}

int orx_batch_set_ban(orx_batch* b, int sid, int ban0, int ban1, int steps, void* stream) {
  return guard([&] {
    need(b, "batch");
    DeviceScope ds(b->device);
    b->b->set_ban(sid, ban0, ban1, steps, S(stream));
  });
}

int orx_batch_next_tokens(orx_batch* b, const int* sids, int n, int* out, void* stream) {
  return guard([&] {
    need(b, "batch");
    if (n <= 0) return;
    need(sids, "sids");
    need(out, "out");
    DeviceScope ds(b->device);
    b->b->next_tokens(sids, n, out, S(stream));
  });
}

int orx_batch_device_error(const orx_batch* b, int* out) {
  return guard([&] {
    need(b, "batch");
    need(out, "out");
    DeviceScope ds(b->device);
    *out = b->b->device_error();
  });
}

int orx_layer32_create(const orx_config* cfg, orx_layer32** out) {
  return guard([&] {
    need(cfg, "cfg");
    need(out, "out");
    *out = nullptr;
    if (cfg->hidden_size != orx::kHidden || cfg->num_q_heads != orx::kQHeads ||
        cfg->num_kv_heads != orx::kKvHeads || cfg->head_dim != orx::kHeadDim ||
        cfg->intermediate_size != orx::kInter)
      throw std::invalid_argument("only the Qwen3-ASR-1.7B head geometry is supported");
    auto* h = new orx_layer32;
    try {
      orx::check(cudaGetDevice(&h->device), "cudaGetDevice");
      h->l = orx::layer32_create(cfg->max_seq_len, cfg->rms_norm_eps, cfg->rope_theta);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_layer32_destroy(orx_layer32* l) {
  if (!l) return;
  DeviceScope ds(l->device);
  orx::layer32_destroy(l->l);
  if (l->d_io) cudaFree(l->d_io);
  delete l;
}

int orx_layer32_set_tensor(orx_layer32* l, const char* name, const float* data, size_t numel,
                           int on_device) {
  return guard([&] {
    need(l, "layer");
    need(name, "name");
    need(data, "data");
    DeviceScope ds(l->device);
    orx::layer32_set_tensor(l->l, name, data, numel, on_device != 0);
  });
}

int orx_layer32_init_synthetic(orx_layer32* l, int seed, int layer) {
  return guard([&] {
    need(l, "layer");
    if (layer < 0 || layer > 4000) throw std::invalid_argument("layer index out of range");
    DeviceScope ds(l->device);
    orx::layer32_init_synthetic(l->l, seed, layer);
  });
}

int orx_layer32_forward_device(orx_layer32* l, const float* d_x, int T, int pos0, float* d_out,
                               void* stream) {
  return guard([&] {
    need(l, "layer");
    if (T <= 0) return;
    need(d_x, "x");
    need(d_out, "out");
    DeviceScope ds(l->device);
    orx::layer32_forward(l->l, d_x, T, pos0, d_out, S(stream));
  });
}

int orx_layer32_forward(orx_layer32* l, const float* x, int T, int pos0, float* out, void* stream) {
  return guard([&] {
    need(l, "layer");
    if (T <= 0) return;
    need(x, "x");
    need(out, "out");
    DeviceScope ds(l->device);
    if (T > l->cap) {
      if (l->d_io) cudaFree(l->d_io);
      l->d_io = nullptr;
      l->cap = 0;
      orx::check(cudaMalloc(&l->d_io, (size_t)2 * T * orx::kHidden * 4), "cudaMalloc");
      l->cap = T;
    }
    const size_t n = (size_t)T * orx::kHidden;
    float* din = l->d_io;
    float* dout = l->d_io + (size_t)l->cap * orx::kHidden;
    orx::check(cudaMemcpyAsync(din, x, n * 4, cudaMemcpyHostToDevice, S(stream)), "cudaMemcpyAsync");
    orx::layer32_forward(l->l, din, T, pos0, dout, S(stream));
    orx::check(cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, S(stream)), "cudaMemcpyAsync");
    orx::check(cudaStreamSynchronize(S(stream)), "cudaStreamSynchronize");
  });
}

int orx_layer32_cache_len(const orx_layer32* l, int* out) {
  return guard([&] {
    need(l, "layer");
    need(out, "out");
    *out = orx::layer32_len(l->l);
  });
}

int orx_layer32_truncate(orx_layer32* l, int len) {
  return guard([&] {
    need(l, "layer");
    orx::layer32_truncate(l->l, len);
  });
}

}  // extern "C"

namespace {
// One device error word per device for the GEMM's bounded waits (made on
// first use, thread-safe).
int* gemm_err_word() {
  static std::mutex mu;
  static int* err_of[64] = {};
  int dev = 0;
  orx::check(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  int*& e = err_of[dev & 63];
  if (!e) {
    orx::check(cudaMalloc(&e, sizeof(int)), "cudaMalloc");
    orx::check(cudaMemset(e, 0, sizeof(int)), "cudaMemset");
  }
  return e;
}

void linear_pre(const uint16_t* in_bf16, const uint16_t* W_bf16, const float* bias,
                float* out_f32, int M, int K, int N, int act, cudaStream_t s) {
  if (act < 0 || act > 2) throw std::invalid_argument("act must be 0 (none), 1 (GELU) or 2 (ReLU)");
  if (reinterpret_cast<uintptr_t>(in_bf16) % 2 || reinterpret_cast<uintptr_t>(W_bf16) % 2 ||
      reinterpret_cast<uintptr_t>(out_f32) % 4 || reinterpret_cast<uintptr_t>(bias) % 4)
    throw std::invalid_argument("misaligned operand (bf16 needs 2-byte, fp32 4-byte alignment)");
  if (K % 8 != 0 || !orx::tc_available() ||
      reinterpret_cast<uintptr_t>(in_bf16) % 16 != 0 || reinterpret_cast<uintptr_t>(W_bf16) % 16 != 0) {
    // shapes a tensor map cannot describe (rows must be 16-byte multiples)
    orx::op_linear_simt(in_bf16, W_bf16, bias, out_f32, M, K, N, act, s);
    orx::check(cudaGetLastError(), "linear");
    return;
  }
  orx::TcArgs g = {};
  g.N = N;
  g.K = K;
  g.T = M;
  g.epi = orx::kEpiLinear;
  g.out_f32 = out_f32;
  g.ldo = N;
  g.err = gemm_err_word();
  g.bias = bias;
  g.act = act;
  orx::launch_gemm_tc(in_bf16, W_bf16, g, 1, s);
  orx::check(cudaGetLastError(), "tcgen05 gemm");
}

// The bf16 copy of Linear's fp32 input, one buffer per calling thread (as
// the reference keeps it, asr_gemm.cu:24-44), grown on demand.
struct CastScratch {
  uint16_t* p = nullptr;
  long long cap = 0;
  int dev = -1;
  ~CastScratch() {
    if (p) cudaFree(p);
  }
};
thread_local CastScratch g_cast;
}  // namespace

extern "C" {

int orx_linear_pre(const uint16_t* in_bf16, const uint16_t* W_bf16, const float* bias,
                   float* out_f32, int M, int K, int N, int act, void* stream) {
  return guard([&] {
    if (M <= 0 || K <= 0 || N <= 0) return;  // empty input is a no-op, as in the reference
    need(in_bf16, "in");
    need(W_bf16, "W");
    need(out_f32, "out");
    linear_pre(in_bf16, W_bf16, bias, out_f32, M, K, N, act, S(stream));
  });
}

int orx_linear(const float* in_f32, const uint16_t* W_bf16, const float* bias, float* out_f32,
               int M, int K, int N, int act, void* stream) {
  return guard([&] {
    if (M <= 0 || K <= 0 || N <= 0) return;
    need(in_f32, "in");
    need(W_bf16, "W");
    need(out_f32, "out");
    const long long n = static_cast<long long>(M) * K;
    int dev = 0;
    orx::check(cudaGetDevice(&dev), "cudaGetDevice");
    if (n > g_cast.cap || dev != g_cast.dev) {
      // the previous buffer may still feed queued work of this thread
      if (g_cast.p) {
        orx::check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        cudaFree(g_cast.p);
        g_cast.p = nullptr;
      }
      orx::check(cudaMalloc(&g_cast.p, sizeof(uint16_t) * (n + 8)), "cudaMalloc");
      g_cast.cap = n;
      g_cast.dev = dev;
    }
    orx::launch_f32_to_bf16(in_f32, g_cast.p, n, S(stream));
    orx::check(cudaGetLastError(), "f32 -> bf16");
    linear_pre(g_cast.p, W_bf16, bias, out_f32, M, K, N, act, S(stream));
  });
}

int orx_f32_to_bf16(const float* in, uint16_t* out, long long n, void* stream) {
  return guard([&] {
    if (n <= 0) return;
    need(in, "in");
    need(out, "out");
    orx::launch_f32_to_bf16(in, out, n, S(stream));
    orx::check(cudaGetLastError(), "f32 -> bf16");
  });
}

int orx_bf16_to_f32(const uint16_t* in, float* out, long long n, void* stream) {
  return guard([&] {
    if (n <= 0) return;
    need(in, "in");
    need(out, "out");
    orx::launch_bf16_to_f32(in, out, n, S(stream));
    orx::check(cudaGetLastError(), "bf16 -> f32");
  });
}

int orx_rms_norm(const float* x, const float* weight, float* out, int rows, int dim, float eps,
                 void* stream) {
  return guard([&] {
    if (rows <= 0 || dim <= 0) return;
    need(x, "x");
    need(weight, "weight");
    need(out, "out");
    orx::op_rms_norm(x, weight, out, rows, dim, eps, S(stream));
    orx::check(cudaGetLastError(), "rms_norm");
  });
}

static int rope(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                float theta, bool half, void* stream) {
  return guard([&] {
    if (n_tokens <= 0 || n_heads <= 0 || head_dim <= 0) return;
    need(x, "x");
    need(positions, "positions");
    if (head_dim % 2) throw std::invalid_argument("head_dim must be even");
    if (n_heads > 65535) throw std::invalid_argument("too many heads");
    orx::op_rope(x, positions, n_tokens, n_heads, head_dim, theta, half, S(stream));
    orx::check(cudaGetLastError(), "rope");
  });
}

int orx_rope_half(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                  float theta_base, void* stream) {
  return rope(x, positions, n_tokens, n_heads, head_dim, theta_base, true, stream);
}

int orx_rope_interleaved(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                         float theta_base, void* stream) {
  return rope(x, positions, n_tokens, n_heads, head_dim, theta_base, false, stream);
}

int orx_swiglu(const float* gate, const float* up, float* out, long long n, void* stream) {
  return guard([&] {
    if (n <= 0) return;
    need(gate, "gate");
    need(up, "up");
    need(out, "out");
    orx::op_swiglu(gate, up, out, n, S(stream));
    orx::check(cudaGetLastError(), "swiglu");
  });
}

int orx_gqa_attention(const float* q, const float* k, const float* v, float* out, int T, int Hq,
                      int Hkv, int head_dim, float scale, int causal, void* stream) {
  return guard([&] {
    if (T <= 0 || Hq <= 0 || Hkv <= 0 || head_dim <= 0) return;
    need(q, "q");
    need(k, "k");
    need(v, "v");
    need(out, "out");
    if (Hq % Hkv) throw std::invalid_argument("Hq must be a multiple of Hkv");
    if (head_dim > 1024) throw std::invalid_argument("head_dim must be <= 1024");
    if (Hkv > 65535) throw std::invalid_argument("too many kv heads");
    orx::check(orx::op_gqa_attention(q, k, v, out, T, Hq, Hkv, head_dim, scale, causal != 0,
                                     S(stream)),
               "gqa attention");
  });
}

int orx_argmax_banned(const float* logits, int n, int ban0, int ban1, int* d_out, void* stream) {
  return guard([&] {
    if (n <= 0) return;  // as in the reference: nothing is written
    need(logits, "logits");
    need(d_out, "out");
    orx::op_argmax_banned(logits, n, ban0, ban1, d_out, S(stream));
    orx::check(cudaGetLastError(), "argmax");
  });
}

int orx_vad_create(int streams, orx_vad** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    auto* h = new orx_vad;
    try {
      cudaGetDevice(&h->device);
      h->v = new orx::BatchVad(streams);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_vad_destroy(orx_vad* v) {
  if (!v) return;
  DeviceScope ds(v->device);
  delete v->v;
  delete v;
}

int orx_vad_set_tensor(orx_vad* v, const char* name, const float* data, size_t numel) {
  return guard([&] {
    need(v, "vad");
    need(name, "name");
    need(data, "data");
    v->v->set_tensor(name, data, numel);
  });
}

int orx_vad_init_synthetic(orx_vad* v, int seed) {
  return guard([&] {
    need(v, "vad");
    DeviceScope ds(v->device);
    v->v->init_synthetic(seed);
  });
}

int orx_vad_reset(orx_vad* v) {
  return guard([&] {
    need(v, "vad");
    DeviceScope ds(v->device);
    v->v->reset();
  });
}

int orx_vad_run(orx_vad* v, const float* pcm, int steps, float* probs, int on_device,
                void* stream) {
  return guard([&] {
    need(v, "vad");
    if (steps < 0) throw std::invalid_argument("negative step count");
    if (steps == 0) return;
    need(pcm, "pcm");
    need(probs, "probs");
    DeviceScope ds(v->device);
    if (on_device) v->v->run_device(pcm, steps, probs, S(stream));
    else v->v->run_host(pcm, steps, probs, S(stream));
  });
}

int orx_synth_f32(float* d_out, long long n, int seed, int tid, double std, float mean,
                  int round_bf16, void* stream) {
  return guard([&] {
    if (n > 0) need(d_out, "d_out");
    if (n <= 0) return;
    orx::launch_synth_f32(d_out, n, seed, tid, std, mean, round_bf16, S(stream));
    orx::check(cudaGetLastError(), "synth");
  });
}

int orx_tower_create(int layers, int windowed, orx_tower** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    auto* h = new orx_tower;
    try {
      orx::check(cudaGetDevice(&h->device), "cudaGetDevice");
      h->t = new orx::AudioTower(layers, windowed != 0);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_tower_destroy(orx_tower* t) {
  if (!t) return;
  DeviceScope ds(t->device);
  delete t->t;
  delete t;
}

int orx_tower_set_tensor(orx_tower* t, const char* name, const void* data, int dtype,
                         size_t numel) {
  return guard([&] {
    need(t, "tower");
    need(name, "name");
    need(data, "data");
    DeviceScope ds(t->device);
    t->t->set_tensor(name, data, dtype, numel);
  });
}

int orx_tower_load_safetensors(orx_tower* t, const char* dir) {
  return guard([&] {
    need(t, "tower");
    need(dir, "model_dir");
    DeviceScope ds(t->device);
    orx::ShardedCheckpoint ck(dir);
    for (const auto& kv : ck.tensors()) {
      if (kv.first.rfind("thinker.audio_tower.", 0) != 0) continue;
      const auto& v = kv.second;
      int dtype;
      size_t es;
      if (v.dtype == "BF16") { dtype = 1; es = 2; }
      else if (v.dtype == "F32") { dtype = 0; es = 4; }
      else throw std::invalid_argument("unsupported dtype " + v.dtype + " for " + kv.first);
      // layers beyond the configured count are not part of this tower
      try {
        t->t->set_tensor(kv.first, v.data, dtype, v.nbytes / es);
      } catch (const std::invalid_argument& e) {
        if (std::string(e.what()).rfind("unknown audio tower tensor", 0) != 0) throw;
      }
    }
    if (!t->t->complete()) throw std::invalid_argument("checkpoint is missing audio tower tensors");
  });
}

int orx_tower_init_synthetic(orx_tower* t, int seed) {
  return guard([&] {
    need(t, "tower");
    DeviceScope ds(t->device);
    t->t->init_synthetic(seed);
  });
}

int orx_tower_weights_complete(const orx_tower* t, int* complete) {
  return guard([&] {
    need(t, "tower");
    need(complete, "complete");
    *complete = t->t->complete() ? 1 : 0;
  });
}

int orx_tower_output_length(int n_frames) { return orx::AudioTower::output_length(n_frames); }

int orx_tower_forward(orx_tower* t, const float* mel, int n_frames, float* out, int* out_tokens,
                      void* stream) {
  return guard([&] {
    need(t, "tower");
    if (n_frames < 0) throw std::invalid_argument("n_frames must be >= 0");
    if (out_tokens) *out_tokens = 0;
    if (n_frames == 0) return;
    need(mel, "mel");
    need(out, "out");
    DeviceScope ds(t->device);
    const int n = t->t->forward_host(mel, n_frames, out, S(stream));
    if (out_tokens) *out_tokens = n;
  });
}

int orx_tower_forward_batch(orx_tower* t, const float* d_mel, const int* frames, int n,
                            float* d_out, int* out_rows, void* stream) {
  return guard([&] {
    need(t, "tower");
    if (n < 0) throw std::invalid_argument("negative utterance count");
    if (out_rows) *out_rows = 0;
    if (n == 0) return;
    need(frames, "frames");
    need(d_mel, "mel");
    need(d_out, "out");
    DeviceScope ds(t->device);
    const int rows = t->t->forward_device(d_mel, frames, n, d_out, S(stream));
    if (out_rows) *out_rows = rows;
  });
}

int orx_sf_create(int conf_layers, int dec_layers, orx_sf** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    auto* h = new orx_sf;
    try {
      orx::check(cudaGetDevice(&h->device), "cudaGetDevice");
      h->s = new orx::Sortformer(conf_layers, dec_layers);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void orx_sf_destroy(orx_sf* s) {
  if (!s) return;
  DeviceScope ds(s->device);
  delete s->s;
  if (s->stage) cudaFree(s->stage);
  delete s;
}

int orx_sf_set_tensor(orx_sf* s, const char* name, const float* data, size_t numel) {
  return guard([&] {
    need(s, "sortformer");
    need(name, "name");
    need(data, "data");
    DeviceScope ds(s->device);
    s->s->set_tensor(name, data, numel, false);
  });
}

int orx_sf_load_safetensors(orx_sf* s, const char* path) {
  return guard([&] {
    need(s, "sortformer");
    need(path, "path");
    DeviceScope ds(s->device);
    s->s->load_safetensors(path);
  });
}

int orx_sf_init_synthetic(orx_sf* s, int seed) {
  return guard([&] {
    need(s, "sortformer");
    DeviceScope ds(s->device);
    s->s->init_synthetic(seed);
  });
}

int orx_sf_weights_complete(const orx_sf* s, int* complete) {
  return guard([&] {
    need(s, "sortformer");
    need(complete, "complete");
    *complete = s->s->complete() ? 1 : 0;
  });
}

int orx_sf_pre_encode(orx_sf* s, const float* mel, int n_frames, int valid, float* out, int* T_out,
                      int* valid_out, int on_device, void* stream) {
  return guard([&] {
    need(s, "sortformer");
    need(mel, "mel");
    need(out, "out");
    if (n_frames <= 0) throw std::invalid_argument("n_frames must be positive");
    DeviceScope ds(s->device);
    int v2 = 0, T2 = 0;
    if (on_device) {
      T2 = s->s->pre_encode_device(mel, n_frames, valid, out, &v2, S(stream));
    } else {
      auto cl = [](int x) { return (x + 2 - 3) / 2 + 1; };
      const int t2 = cl(cl(cl(n_frames)));
      const size_t nin = (size_t)128 * n_frames, nout = (size_t)t2 * 512;
      float* d = s->ensure(nin + nout);
      orx::check(cudaMemcpyAsync(d, mel, nin * 4, cudaMemcpyHostToDevice, S(stream)), "copy in");
      T2 = s->s->pre_encode_device(d, n_frames, valid, d + nin, &v2, S(stream));
      orx::check(cudaMemcpyAsync(out, d + nin, nout * 4, cudaMemcpyDeviceToHost, S(stream)), "copy out");
      orx::check(cudaStreamSynchronize(S(stream)), "sync");
    }
    if (T_out) *T_out = T2;
    if (valid_out) *valid_out = v2;
  });
}

int orx_sf_forward(orx_sf* s, const float* emb, int T, int valid, float* preds, int on_device,
                   void* stream) {
  return guard([&] {
    need(s, "sortformer");
    need(emb, "emb");
    need(preds, "preds");
    if (T <= 0) throw std::invalid_argument("T must be positive");
    DeviceScope ds(s->device);
    if (on_device) {
      s->s->encode_decode_device(emb, T, valid, preds, S(stream));
    } else {
      const size_t nin = (size_t)T * 512, nout = (size_t)T * 4;
      float* d = s->ensure(nin + nout);
      orx::check(cudaMemcpyAsync(d, emb, nin * 4, cudaMemcpyHostToDevice, S(stream)), "copy in");
      s->s->encode_decode_device(d, T, valid, d + nin, S(stream));
      orx::check(cudaMemcpyAsync(preds, d + nin, nout * 4, cudaMemcpyDeviceToHost, S(stream)), "copy out");
      orx::check(cudaStreamSynchronize(S(stream)), "sync");
    }
  });
}

int orx_sf_step(orx_sf* s, const float* mel, int n_frames, int valid, const float* cache,
                int n_cache, float* preds, int* T_out, int* valid_out, int on_device, void* stream) {
  return guard([&] {
    need(s, "sortformer");
    need(mel, "mel");
    need(preds, "preds");
    if (n_frames <= 0) throw std::invalid_argument("n_frames must be positive");
    if (n_cache < 0) throw std::invalid_argument("n_cache must be >= 0");
    if (n_cache > 0) need(cache, "cache");
    DeviceScope ds(s->device);
    int T = 0, v = 0;
    if (on_device) {
      T = s->s->step_device(mel, n_frames, valid, cache, n_cache, preds, &v, S(stream));
    } else {
      auto cl = [](int x) { return (x + 2 - 3) / 2 + 1; };
      const int tt = n_cache + cl(cl(cl(n_frames)));
      const size_t nin = (size_t)128 * n_frames, nc = (size_t)n_cache * 512, nout = (size_t)tt * 4;
      float* d = s->ensure(nin + nc + nout);
      orx::check(cudaMemcpyAsync(d, mel, nin * 4, cudaMemcpyHostToDevice, S(stream)), "copy in");
      if (nc)
        orx::check(cudaMemcpyAsync(d + nin, cache, nc * 4, cudaMemcpyHostToDevice, S(stream)), "copy in");
      T = s->s->step_device(d, n_frames, valid, d + nin, n_cache, d + nin + nc, &v, S(stream));
      orx::check(cudaMemcpyAsync(preds, d + nin + nc, nout * 4, cudaMemcpyDeviceToHost, S(stream)),
                 "copy out");
      orx::check(cudaStreamSynchronize(S(stream)), "sync");
    }
    if (T_out) *T_out = T;
    if (valid_out) *valid_out = v;
  });
}

}  // extern "C"
