// Model weights on the device and their placement from reference tensors.
#include <cstdlib>
#include <cstring>
#include <regex>

#include "common.cuh"
#include "engine.h"

namespace orx {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ORX_NO_PDL");
    return !(v && v[0] == '1');
  }();
  return on;
}

namespace {
// Tensor slots within a layer, in the order of the synthetic generator's ids.
enum Slot { kInLn, kPostLn, kQNorm, kKNorm, kQ, kK, kV, kO, kGate, kUp, kDown, kSlots };
const char* kSlotNames[kSlots] = {"input_layernorm", "post_attention_layernorm",
                                  "self_attn.q_norm", "self_attn.k_norm",
                                  "self_attn.q_proj", "self_attn.k_proj",
                                  "self_attn.v_proj", "self_attn.o_proj",
                                  "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"};
constexpr int kTidEmbed = 0, kTidFinalNorm = 1, kLayerBase = 16, kLayerStride = 16;

size_t slot_numel(int s) {
  switch (s) {
    case kInLn: case kPostLn: return kHidden;
    case kQNorm: case kKNorm: return kHeadDim;
    case kQ: case kO: return (size_t)kQDim * kHidden;
    case kK: case kV: return (size_t)kKvDim * kHidden;
    case kGate: case kUp: case kDown: return (size_t)kInter * kHidden;
  }
  return 0;
}
}  // namespace

Model::Model(const ModelConfig& c) : cfg(c) {
  if (cfg.num_layers <= 0 || cfg.vocab_size <= 0 || cfg.max_seq_len <= 0)
    throw std::invalid_argument("invalid decoder config");
  int dev = 0;
  ORX_CHECK(cudaGetDevice(&dev));
  ORX_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  embed = dalloc<uint16_t>((size_t)cfg.vocab_size * kHidden);
  final_norm = dalloc<float>(kHidden);
  layers.resize(cfg.num_layers);
  for (auto& L : layers) {
    L.in_ln = dalloc<float>(kHidden);
    L.post_ln = dalloc<float>(kHidden);
    L.q_norm = dalloc<float>(kHeadDim);
    L.k_norm = dalloc<float>(kHeadDim);
    L.qkv = dalloc<uint16_t>((size_t)kQkvDim * kHidden);
    L.o = dalloc<uint16_t>((size_t)kHidden * kQDim);
    L.gateup = dalloc<uint16_t>((size_t)2 * kInter * kHidden);
    L.down = dalloc<uint16_t>((size_t)kHidden * kInter);
  }
  rope_positions = cfg.max_seq_len;
  rope_cos = dalloc<float>((size_t)rope_positions * 64);
  rope_sin = dalloc<float>((size_t)rope_positions * 64);
  launch_rope_table(rope_cos, rope_sin, rope_positions, cfg.rope_theta, 0);
  ORX_CHECK(cudaGetLastError());
  ORX_CHECK(cudaDeviceSynchronize());
  have.assign(2 + (size_t)cfg.num_layers * kSlots, 0);
}

Model::~Model() {
  cudaFree(embed);
  cudaFree(final_norm);
  for (auto& L : layers) {
    for (void* p : {(void*)L.in_ln, (void*)L.post_ln, (void*)L.q_norm, (void*)L.k_norm,
                    (void*)L.qkv, (void*)L.o, (void*)L.gateup, (void*)L.down})
      cudaFree(p);
  }
  cudaFree(rope_cos);
  cudaFree(rope_sin);
}

bool Model::complete() const {
  for (uint8_t h : have)
    if (!h) return false;
  return true;
}

// Placement (mirrors the fusion in asr_text_decoder.cu:296-306, with a
// different gate|up layout): qkv rows = [q 2048 | k 1024 | v 1024]; gate/up
// are interleaved in 128-row tiles [64 gate rows | 64 up rows] so one GEMV
// warp or one GEMM tile sees matching gate and up rows for the SwiGLU
// epilogue. Norm weights are stored fp32 (bf16 inputs upcast exactly, as
// LoadF32 does at asr_text_decoder.cu:219-236).
void Model::set_tensor(const std::string& name, const void* src, int dtype, size_t numel,
                       bool device) {
  static const std::regex re(R"(^thinker\.model\.layers\.(\d+)\.(.+)\.weight$)");
  const cudaMemcpyKind kind = device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  auto put_f32 = [&](float* dst, size_t n) {
    if (numel != n) throw std::invalid_argument("shape mismatch for " + name);
    if (dtype == 0) {
      ORX_CHECK(cudaMemcpy(dst, src, n * 4, kind));
    } else if (device) {
      launch_bf16_to_f32(static_cast<const uint16_t*>(src), dst, (long long)n, 0);
      ORX_CHECK(cudaDeviceSynchronize());
    } else {
      std::vector<float> tmp(n);
      const uint16_t* b = static_cast<const uint16_t*>(src);
      for (size_t i = 0; i < n; ++i) {
        const uint32_t u = static_cast<uint32_t>(b[i]) << 16;
        std::memcpy(&tmp[i], &u, 4);
      }
      ORX_CHECK(cudaMemcpy(dst, tmp.data(), n * 4, cudaMemcpyHostToDevice));
    }
  };
  auto put_bf16 = [&](uint16_t* dst, size_t n, size_t dpitch_rows, size_t block_rows,
                      size_t nblocks) {
    if (numel != n) throw std::invalid_argument("shape mismatch for " + name);
    if (dtype != 1) throw std::invalid_argument("expected BF16 for " + name);
    const size_t width = block_rows * kHidden * 2;
    ORX_CHECK(cudaMemcpy2D(dst, dpitch_rows * kHidden * 2, src, width, width, nblocks, kind));
  };
  if (name == "thinker.model.embed_tokens.weight" || name == "thinker.lm_head.weight") {
    put_bf16(embed, (size_t)cfg.vocab_size * kHidden, cfg.vocab_size, cfg.vocab_size, 1);
    have[0] = 1;
    return;
  }
  if (name == "thinker.model.norm.weight") {
    put_f32(final_norm, kHidden);
    have[1] = 1;
    return;
  }
  std::smatch m;
  if (!std::regex_match(name, m, re)) throw std::invalid_argument("unknown tensor " + name);
  const int l = std::stoi(m[1].str());
  if (l < 0 || l >= cfg.num_layers) throw std::invalid_argument("layer out of range: " + name);
  const std::string sub = m[2].str();
  int s = -1;
  for (int i = 0; i < kSlots; ++i)
    if (sub == kSlotNames[i]) s = i;
  if (s < 0) throw std::invalid_argument("unknown tensor " + name);
  Layer& L = layers[l];
  const size_t n = slot_numel(s);
  switch (s) {
    case kInLn: put_f32(L.in_ln, n); break;
    case kPostLn: put_f32(L.post_ln, n); break;
    case kQNorm: put_f32(L.q_norm, n); break;
    case kKNorm: put_f32(L.k_norm, n); break;
    case kQ: put_bf16(L.qkv, n, kQDim, kQDim, 1); break;
    case kK: put_bf16(L.qkv + (size_t)kQDim * kHidden, n, kKvDim, kKvDim, 1); break;
    case kV: put_bf16(L.qkv + (size_t)(kQDim + kKvDim) * kHidden, n, kKvDim, kKvDim, 1); break;
    case kO: put_bf16(L.o, n, kHidden, kHidden, 1); break;
    case kGate: put_bf16(L.gateup, n, 128, 64, kInter / 64); break;
    case kUp: put_bf16(L.gateup + (size_t)64 * kHidden, n, 128, 64, kInter / 64); break;
    case kDown: {
      if (numel != n || dtype != 1) throw std::invalid_argument("bad tensor " + name);
      ORX_CHECK(cudaMemcpy(L.down, src, n * 2, kind));
      break;
    }
  }
  have[2 + (size_t)l * kSlots + s] = 1;
}

// Seeded synthetic weights, generated on the device; bit-exact with
// oracle/synth.py (matrices N(0,0.02), norms 1 + N(0,0.02), all bf16-rounded).
void Model::init_synthetic(int seed, cudaStream_t s) {
  size_t maxn = (size_t)cfg.vocab_size * kHidden;
  if ((size_t)kInter * kHidden > maxn) maxn = (size_t)kInter * kHidden;
  uint16_t* tmp = dalloc<uint16_t>(maxn);
  float* tmpf = dalloc<float>(kHidden);
  auto gen = [&](const std::string& name, int tid, size_t n, bool norm) {
    if (norm) {
      launch_synth_f32(tmpf, (long long)n, seed, tid, 0.02, 1.0f, 1, s);
      ORX_CHECK(cudaStreamSynchronize(s));
      set_tensor(name, tmpf, 0, n, true);
    } else {
      launch_synth_bf16(tmp, (long long)n, seed, tid, 0.02, 0.0f, s);
      ORX_CHECK(cudaStreamSynchronize(s));
      set_tensor(name, tmp, 1, n, true);
    }
  };
  gen("thinker.model.embed_tokens.weight", kTidEmbed, (size_t)cfg.vocab_size * kHidden, false);
  gen("thinker.model.norm.weight", kTidFinalNorm, kHidden, true);
  for (int l = 0; l < cfg.num_layers; ++l)
    for (int j = 0; j < kSlots; ++j)
      gen("thinker.model.layers." + std::to_string(l) + "." + kSlotNames[j] + ".weight",
          kLayerBase + l * kLayerStride + j, slot_numel(j), j < 4);
  ORX_CHECK(cudaFree(tmp));
  ORX_CHECK(cudaFree(tmpf));
}

KvPool::KvPool(int layers, int pages_) : num_layers(layers), pages(pages_) {
  base = dalloc<uint16_t>((size_t)layers * pages * kPageElems);
  ORX_CHECK(cudaMemset(base, 0, (size_t)layers * pages * kPageElems * 2));
}
KvPool::~KvPool() { cudaFree(base); }

}  // namespace orx
