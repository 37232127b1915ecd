// C entry points over the UNMODIFIED reference decoder, for parity checks only.
//
// TEST INFRASTRUCTURE: compiled by oracle/build_ref.sh together with the
// reference's own sources (src/model/asr_text_decoder.cu, asr_gemm.cu,
// asr_ops.cu, src/gpu/memory.cc, gpu_lock.cc, src/io/safetensor.cc,
// sharded_safetensor.cc, src/core/tensor.cc) into oracle/_ref/libref_asr.so.
// It drives orator::model::AsrTextDecoder exactly as
// test/unit/model/test_asr_decoder.cc:46-51 does.  The product never links it.
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "io/sharded_safetensor.h"
#include "model/asr_text_decoder.h"

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

void* ref_create(const char* model_dir, int num_layers, int vocab, int max_seq) {
  try {
    auto* h = new RefHandle;
    orator::model::AsrTextConfig c;
    c.num_layers = num_layers;
    c.vocab_size = vocab;
    c.max_seq_len = max_seq;
    c.cuda_graph_enabled = false;
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

void ref_truncate(void* p, int len) { static_cast<RefHandle*>(p)->dec->TruncateCache(len); }
int ref_cache_len(void* p) { return static_cast<RefHandle*>(p)->dec->cache_len(); }

}  // extern "C"
