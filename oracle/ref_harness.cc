// C entry points over the UNMODIFIED reference decoder, for parity checks only.
//
// TEST INFRASTRUCTURE: compiled by oracle/build_ref.sh together with the
// reference's own sources (src/model/asr_text_decoder.cu, asr_gemm.cu,
// asr_ops.cu, src/gpu/memory.cc, gpu_lock.cc, src/io/safetensor.cc,
// sharded_safetensor.cc, src/core/tensor.cc) into oracle/_ref/libref_asr.so.
// It drives orator::model::AsrTextDecoder exactly as
// test/unit/model/test_asr_decoder.cc:46-51 does.  The product never links it.
#include <cmath>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "io/sharded_safetensor.h"
#include "model/asr_audio_tower.h"
#include "model/asr_gemm.h"
#include "model/asr_ops.cuh"
#include "model/asr_text_decoder.h"
#include "model/conformer_layer.h"
#include "model/conformer_preencode.h"
#include "model/sortformer_decoder.h"
#include "io/safetensor.h"
#include "pipeline/gpu_vad.h"

namespace {
struct RefHandle {
  std::unique_ptr<orator::io::ShardedSafeTensors> w;
  std::unique_ptr<orator::model::AsrTextDecoder> dec;
  int* d_tok = nullptr;
};
thread_local std::string g_err;
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

static void* create(const char* model_dir, int num_layers, int vocab, int max_seq, bool graphs) {
  try {
    auto* h = new RefHandle;
    orator::model::AsrTextConfig c;
    c.num_layers = num_layers;
    c.vocab_size = vocab;
    c.max_seq_len = max_seq;
    c.cuda_graph_enabled = graphs;
    h->w = std::make_unique<orator::io::ShardedSafeTensors>(model_dir);
    h->dec = std::make_unique<orator::model::AsrTextDecoder>(c);
    h->dec->LoadWeights(*h->w);
    if (cudaMalloc(&h->d_tok, sizeof(int)) != cudaSuccess) throw std::runtime_error("malloc");
    return h;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void* ref_create(const char* model_dir, int num_layers, int vocab, int max_seq) {
  return create(model_dir, num_layers, vocab, max_seq, false);
}

// As ref_create, with the reference's CUDA-graph decode loop enabled (its
// default AsrTextConfig, the fastest path of DecodeGreedy).
void* ref_create_graphs(const char* model_dir, int num_layers, int vocab, int max_seq) {
  return create(model_dir, num_layers, vocab, max_seq, true);
}

// Times one DecodeGreedy(start_pos, max_new, no EOS, no ban, batch) call:
// *ms = elapsed time between CUDA events on the legacy stream around the
// call (DecodeGreedy synchronizes before returning), *n_out = tokens made.
int ref_time_greedy(void* p, int start_pos, int max_new, int batch, float* ms, int* n_out) {
  try {
    auto* h = static_cast<RefHandle*>(p);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaDeviceSynchronize();
    cudaEventRecord(a, 0);
    auto v = h->dec->DecodeGreedy(start_pos, max_new, -1, -1, 0, batch);
    cudaEventRecord(b, 0);
    cudaEventSynchronize(b);
    cudaEventElapsedTime(ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    *n_out = static_cast<int>(v.size());
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

void ref_destroy(void* p) {
  auto* h = static_cast<RefHandle*>(p);
  if (!h) return;
  cudaFree(h->d_tok);
  delete h;
}

int ref_prefill_at(void* p, const float* embeds, int T, int pos0) {
  try {
    static_cast<RefHandle*>(p)->dec->PrefillAt(embeds, T, pos0);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

int ref_copy_logits(void* p, float* out) {
  try {
    auto v = static_cast<RefHandle*>(p)->dec->CopyLogits();
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

int ref_argmax(void* p, int ban0, int ban1) {
  return static_cast<RefHandle*>(p)->dec->Argmax(ban0, ban1);
}

// One teacher-forced decode step: embed `tok` on the device, forward at `pos`.
int ref_decode_step_token(void* p, int tok, int pos) {
  auto* h = static_cast<RefHandle*>(p);
  if (cudaMemcpy(h->d_tok, &tok, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return 1;
  try {
    h->dec->DecodeStepDevice(h->d_tok, pos);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

int ref_decode_greedy(void* p, int start_pos, int max_new, int eos0, int eos1,
                      int ban_steps, int batch, int* out, int* n_out) {
  try {
    auto v = static_cast<RefHandle*>(p)->dec->DecodeGreedy(start_pos, max_new, eos0, eos1,
                                                           ban_steps, batch);
    std::memcpy(out, v.data(), v.size() * sizeof(int));
    *n_out = static_cast<int>(v.size());
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

// ---- the reference's free operators on device pointers (asr_ops.cuh:24-62,
// asr_gemm.h:24-41), called unmodified; the caller owns every buffer. Each
// returns 0 after a device synchronize, 1 on an exception or CUDA error.
#define REF_OP(body)                                           \
  try {                                                        \
    body;                                                      \
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 1;     \
  } catch (const std::exception& e) {                          \
    g_err = e.what();                                          \
    return 1;                                                  \
  }
namespace ops = orator::model::asr_ops;
namespace gm = orator::model::asr_gemm;
int ref_op_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps) {
  REF_OP(ops::RmsNorm(x, w, out, rows, dim, eps))
}
int ref_op_rope_half(float* x, const int* pos, int n, int heads, int dim, float theta) {
  REF_OP(ops::RopeHalf(x, pos, n, heads, dim, theta))
}
int ref_op_rope_interleaved(float* x, const int* pos, int n, int heads, int dim, float theta) {
  REF_OP(ops::RopeInterleaved(x, pos, n, heads, dim, theta))
}
int ref_op_swiglu(const float* g, const float* u, float* out, int n) {
  REF_OP(ops::SwiGLU(g, u, out, n))
}
int ref_op_gqa(const float* q, const float* k, const float* v, float* out, int T, int hq,
               int hkv, int dh, float scale, int causal) {
  REF_OP(ops::GqaAttention(q, k, v, out, T, hq, hkv, dh, scale, causal != 0))
}
int ref_op_argmax_banned(const float* x, int n, int ban0, int ban1, int* out) {
  REF_OP(ops::ArgmaxBanned(x, n, ban0, ban1, out))
}
int ref_op_f32_to_bf16(const float* in, uint16_t* out, long n) { REF_OP(gm::F32ToBf16(in, out, n)) }
int ref_op_bf16_to_f32(const uint16_t* in, float* out, long n) { REF_OP(gm::Bf16ToF32(in, out, n)) }
int ref_op_linear(const float* in, const uint16_t* w, const float* bias, float* out, int M, int K,
                  int N, int act) {
  REF_OP(gm::Linear(in, w, bias, out, M, K, N, act))
}
int ref_op_linear_pre(const uint16_t* in, const uint16_t* w, const float* bias, float* out, int M,
                      int K, int N, int act) {
  REF_OP(gm::LinearPre(in, w, bias, out, M, K, N, act))
}

// ---- the reference's audio tower (src/model/asr_audio_tower.cu) ----
struct RefTower {
  std::unique_ptr<orator::io::ShardedSafeTensors> w;
  std::unique_ptr<orator::model::AsrAudioTower> t;
};
void* ref_tower_create(const char* model_dir, int layers, int windowed) {
  try {
    auto* h = new RefTower;
    orator::model::AsrAudioConfig c;
    c.encoder_layers = layers;
    c.windowed_attention = windowed != 0;
    h->w = std::make_unique<orator::io::ShardedSafeTensors>(model_dir);
    h->t = std::make_unique<orator::model::AsrAudioTower>(c);
    h->t->LoadWeights(*h->w);
    return h;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void ref_tower_destroy(void* h) { delete static_cast<RefTower*>(h); }
// mel [128, n_frames] (host) -> out [N, 2048] (host, room for
// OutputLength(n_frames) rows); returns N, or -1.
int ref_tower_forward(void* h, const float* mel, int n_frames, float* out) {
  try {
    int n = 0;
    auto v = static_cast<RefTower*>(h)->t->Forward(mel, n_frames, &n);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return n;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
int ref_tower_output_length(int n_frames) {
  return orator::model::AsrAudioTower::OutputLength(n_frames);
}

// ---- the reference's GPU speech detector (src/pipeline/gpu_vad.cu) ----
void* ref_gpuvad_create(const char* weights_path) {
  try {
    orator::pipeline::GpuVad::Params p;
    p.silero_model_path = weights_path;
    return new orator::pipeline::GpuVad(p);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void ref_gpuvad_destroy(void* h) { delete static_cast<orator::pipeline::GpuVad*>(h); }
// Per-window probabilities of n samples from a fresh state (DebugWindowProbs).
int ref_gpuvad_probs(void* h, const float* pcm, int n, float* out) {
  try {
    auto v = static_cast<orator::pipeline::GpuVad*>(h)->DebugWindowProbs(pcm, n);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return static_cast<int>(v.size());
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
void ref_gpuvad_reset(void* h) { static_cast<orator::pipeline::GpuVad*>(h)->Reset(); }
// Push samples and drain finished speech segments: pairs (start, end) into
// out[2 * cap]; returns the number of segments.
int ref_gpuvad_push_drain(void* h, const float* pcm, int n, int finalize, long* out, int cap) {
  try {
    auto* v = static_cast<orator::pipeline::GpuVad*>(h);
    v->Push(pcm, n);
    std::vector<orator::core::VadSegmentResult> segs;
    v->DrainSegments(finalize != 0, &segs);
    int k = 0;
    for (const auto& s : segs) {
      if (k >= cap) break;
      out[2 * k] = s.start_sample;
      out[2 * k + 1] = s.end_sample;
      ++k;
    }
    return k;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

void ref_truncate(void* p, int len) { static_cast<RefHandle*>(p)->dec->TruncateCache(len); }
int ref_cache_len(void* p) { return static_cast<RefHandle*>(p)->dec->cache_len(); }

// ---- the reference's Sortformer network pieces (conformer_preencode.cu,
// conformer_layer.cu, sortformer_decoder.cu), assembled as
// SortformerDiarizer::ForwardEncoderDecoder does
// (src/model/streaming_sortformer.cc:391-418) ----
struct RefSortformer {
  std::unique_ptr<orator::io::SafeTensorReader> r;
  std::unique_ptr<orator::model::ConformerPreEncode> pre;
  std::vector<std::unique_ptr<orator::model::ConformerLayer>> layers;
  std::unique_ptr<orator::model::SortformerDecoder> dec;
  float* dx = nullptr;
  float* dpe = nullptr;
  size_t cap = 0;
};
void* ref_sf_create(const char* path, int conf_layers, int dec_layers) {
  try {
    auto* h = new RefSortformer;
    h->r = std::make_unique<orator::io::SafeTensorReader>(path);
    h->pre = std::make_unique<orator::model::ConformerPreEncode>();
    h->pre->LoadWeights(*h->r);
    for (int l = 0; l < conf_layers; ++l) {
      auto layer = std::make_unique<orator::model::ConformerLayer>(512);
      layer->LoadWeights(*h->r, "encoder.layers." + std::to_string(l));
      h->layers.push_back(std::move(layer));
    }
    h->dec = std::make_unique<orator::model::SortformerDecoder>(512, 192, 8, 768, dec_layers, 4);
    h->dec->LoadWeights(*h->r);
    return h;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void ref_sf_destroy(void* p) {
  auto* h = static_cast<RefSortformer*>(p);
  if (h->dx) cudaFree(h->dx);
  if (h->dpe) cudaFree(h->dpe);
  delete h;
}
// mel [n_mels, n_frames] (host, freq-major) -> out [T2, 512] (host); writes
// T2 and the valid length; returns 0 or -1.
int ref_sf_preencode(void* p, const float* mel, int n_mels, int n_frames, int valid, float* out,
                     int* T2, int* valid2) {
  try {
    auto v = static_cast<RefSortformer*>(p)->pre->Forward(mel, n_mels, n_frames, valid, T2,
                                                          valid2, nullptr);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
// ForwardEncoderDecoder: emb [T, 512] (host) -> preds [T, 4] (host).
int ref_sf_encdec(void* p, const float* emb, int T, int valid, float* preds) {
  try {
    auto* h = static_cast<RefSortformer*>(p);
    const int D = 512;
    const float xscale = std::sqrt(static_cast<float>(D));
    std::vector<float> xin(static_cast<size_t>(T) * D);
    for (size_t i = 0; i < xin.size(); ++i) xin[i] = emb[i] * xscale;
    std::vector<float> pe = orator::model::ConformerLayer::BuildPosEmb(T, D);
    if (xin.size() + pe.size() > h->cap) {
      if (h->dx) cudaFree(h->dx);
      if (h->dpe) cudaFree(h->dpe);
      cudaMalloc(&h->dx, xin.size() * 4);
      cudaMalloc(&h->dpe, pe.size() * 4);
      h->cap = xin.size() + pe.size();
    }
    cudaMemcpy(h->dx, xin.data(), xin.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(h->dpe, pe.data(), pe.size() * 4, cudaMemcpyHostToDevice);
    for (auto& l : h->layers) l->Forward(h->dx, T, valid, h->dpe, nullptr);
    auto pr = h->dec->Forward(h->dx, T, valid, nullptr);
    for (int f = valid; f < T; ++f)
      for (int s = 0; s < 4; ++s) pr[static_cast<size_t>(f) * 4 + s] = 0.0f;
    std::memcpy(preds, pr.data(), pr.size() * sizeof(float));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

}  // extern "C"
