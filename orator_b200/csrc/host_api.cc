// C++ host classes (include/orator_b200/asr_text_decoder.h) over the C ABI.
#include "orator_b200/asr_text_decoder.h"

namespace orator {
namespace model {
namespace {

void Check(int rc) {
  if (rc == ORX_OK) return;
  if (rc == ORX_ECUDA) throw GpuError(orx_last_error());
  throw std::runtime_error(orx_last_error());
}

}  // namespace

AsrTextDecoder::AsrTextDecoder(const AsrTextConfig& c) : config_(c) {
  orx_config oc;
  orx_config_default(&oc);
  oc.hidden_size = c.hidden_size;
  oc.num_layers = c.num_layers;
  oc.num_q_heads = c.num_q_heads;
  oc.num_kv_heads = c.num_kv_heads;
  oc.head_dim = c.head_dim;
  oc.intermediate_size = c.intermediate_size;
  oc.vocab_size = c.vocab_size;
  oc.rms_norm_eps = c.rms_norm_eps;
  oc.rope_theta = c.rope_theta;
  oc.max_seq_len = c.max_seq_len;
  oc.profile = c.profile ? 1 : 0;
  oc.cuda_graph_enabled = c.cuda_graph_enabled ? 1 : 0;
  Check(orx_decoder_create(&oc, &h_));
}

AsrTextDecoder::~AsrTextDecoder() { orx_decoder_destroy(h_); }

void AsrTextDecoder::LoadWeights(const std::string& model_dir) {
  Check(orx_decoder_load_safetensors(h_, model_dir.c_str()));
}

void AsrTextDecoder::SetTensor(const std::string& name, const void* data, bool bf16, size_t numel,
                               bool on_device) {
  Check(orx_decoder_set_tensor(h_, name.c_str(), data, bf16 ? 1 : 0, numel, on_device ? 1 : 0));
}

void AsrTextDecoder::InitSynthetic(int seed) { Check(orx_decoder_init_synthetic(h_, seed)); }

void AsrTextDecoder::ResetCache() { Check(orx_decoder_reset_cache(h_)); }

void AsrTextDecoder::Embed(int token_id, float* out) const {
  Check(orx_decoder_embed(h_, token_id, out));
}

void AsrTextDecoder::Prefill(const float* embeds, int T, cudaStream_t stream) {
  PrefillAt(embeds, T, 0, stream);
}

void AsrTextDecoder::PrefillAt(const float* embeds, int T, int pos0, cudaStream_t stream) {
  Check(orx_decoder_prefill_at(h_, embeds, T, pos0, stream));
}

void AsrTextDecoder::TruncateCache(int len) { Check(orx_decoder_truncate_cache(h_, len)); }

int AsrTextDecoder::cache_len() const {
  int n = 0;
  Check(orx_decoder_cache_len(h_, &n));
  return n;
}

void AsrTextDecoder::DecodeStep(const float* embed, int pos, cudaStream_t stream) {
  Check(orx_decoder_decode_step(h_, embed, pos, stream));
}

void AsrTextDecoder::DecodeStepDevice(const int* d_token, int pos, cudaStream_t stream) {
  Check(orx_decoder_decode_step_device(h_, d_token, pos, stream));
}

int AsrTextDecoder::Argmax(int ban0, int ban1, cudaStream_t stream) {
  int t = 0;
  Check(orx_decoder_argmax(h_, ban0, ban1, stream, &t));
  return t;
}

void AsrTextDecoder::ArgmaxToDevice(int* d_out, int ban0, int ban1, cudaStream_t stream) {
  Check(orx_decoder_argmax_to_device(h_, d_out, ban0, ban1, stream));
}

int AsrTextDecoder::ReadTokenId(const int* d_token, cudaStream_t stream) const {
  int t = 0;
  Check(orx_decoder_read_token_id(h_, d_token, stream, &t));
  return t;
}

std::vector<int> AsrTextDecoder::DecodeGreedy(int start_pos, int max_new, int eos0, int eos1,
                                              int ban_steps, int batch, cudaStream_t stream) {
  std::vector<int> out(max_new > 0 ? max_new : 0);
  int n = 0;
  Check(orx_decoder_decode_greedy(h_, start_pos, max_new, eos0, eos1, ban_steps, batch, stream,
                                  out.data(), &n));
  out.resize(n);
  return out;
}

std::vector<float> AsrTextDecoder::CopyLogits() const {
  std::vector<float> out(config_.vocab_size);
  Check(orx_decoder_copy_logits(h_, out.data()));
  return out;
}

AsrSessionPool::AsrSessionPool(const AsrTextDecoder& weights, int max_sessions, int max_batch,
                               int pool_pages, int max_pages_per_session) {
  Check(orx_batch_create(weights.handle(), max_sessions, max_batch, pool_pages,
                         max_pages_per_session, &h_));
}

AsrSessionPool::~AsrSessionPool() { orx_batch_destroy(h_); }

int AsrSessionPool::CreateSession() {
  int sid = -1;
  Check(orx_batch_session_create(h_, &sid));
  return sid;
}

void AsrSessionPool::FreeSession(int session) { Check(orx_batch_session_free(h_, session)); }

void AsrSessionPool::PrefillAt(int session, const float* embeds, int T, cudaStream_t stream) {
  Check(orx_batch_prefill(h_, &session, &T, 1, embeds, stream));
}

void AsrSessionPool::PrefillAt(const std::vector<int>& sessions, const std::vector<int>& lens,
                               const float* embeds, cudaStream_t stream) {
  if (sessions.size() != lens.size()) throw std::runtime_error("sessions and lens differ in size");
  Check(orx_batch_prefill(h_, sessions.data(), lens.data(), static_cast<int>(sessions.size()),
                          embeds, stream));
}

std::vector<int> AsrSessionPool::StepAll(const std::vector<int>& sessions, cudaStream_t stream) {
  std::vector<int> out(sessions.size());
  Check(orx_batch_step(h_, sessions.data(), static_cast<int>(sessions.size()), out.data(), stream));
  return out;
}

std::vector<int> AsrSessionPool::PendingTokens(const std::vector<int>& sessions,
                                               cudaStream_t stream) {
  std::vector<int> out(sessions.size());
  Check(orx_batch_next_tokens(h_, sessions.data(), static_cast<int>(sessions.size()), out.data(),
                              stream));
  return out;
}

void AsrSessionPool::SetBan(int session, int ban0, int ban1, int steps, cudaStream_t stream) {
  Check(orx_batch_set_ban(h_, session, ban0, ban1, steps, stream));
}

void AsrSessionPool::TruncateCache(int session, int len) {
  Check(orx_batch_truncate(h_, session, len));
}

int AsrSessionPool::cache_len(int session) const {
  int n = 0;
  Check(orx_batch_cache_len(h_, session, &n));
  return n;
}

int AsrSessionPool::free_pages() const {
  int n = 0;
  Check(orx_batch_free_pages(h_, &n));
  return n;
}

}  // namespace model
}  // namespace orator
