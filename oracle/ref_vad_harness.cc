// C entry points over the reference's CPU speech detector (AsrSileroVad,
// test/utils/asr_vad_cpu.cc, "the reference of record the GPU detector is
// gated against"), for parity checks only.
//
// TEST INFRASTRUCTURE: compiled by oracle/build_ref.sh with the reference's
// own sources into oracle/_ref/libref_vad_cpu.so. The product never links it.
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "asr_vad_cpu.h"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char* ref_vadcpu_last_error() { return g_err.c_str(); }

void* ref_vadcpu_create(const char* weights_path) {
  try {
    orator::pipeline::AsrSileroVad::Params p;
    p.silero_model_path = weights_path;
    return new orator::pipeline::AsrSileroVad(p);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void ref_vadcpu_destroy(void* h) { delete static_cast<orator::pipeline::AsrSileroVad*>(h); }

// Per-window speech probabilities of `n` samples from a fresh state.
int ref_vadcpu_probs(void* h, const float* pcm, int n, float* out) {
  auto v = static_cast<orator::pipeline::AsrSileroVad*>(h)->DebugWindowProbs(pcm, n);
  std::memcpy(out, v.data(), v.size() * sizeof(float));
  return static_cast<int>(v.size());
}

}  // extern "C"
