/* C ABI of the B200 Qwen3-ASR text-decoder library (liborator_b200.so).
 *
 * Plain pointers, sizes and status codes; no C++ or torch types cross it.
 * Every call returns ORX_OK (0) or an error code; orx_last_error() gives the
 * message of the last failure on the calling thread.  Streams are passed as
 * `void*` holding a cudaStream_t (NULL = legacy default stream).
 *
 * Each entry point names the reference interface it replaces
 * (thomas-hiddenpeak/Orator, path:line).
 */
#ifndef ORX_H_
#define ORX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORX_OK 0
#define ORX_EINVAL 1 /* bad argument or state (std::runtime_error in the reference) */
#define ORX_ECUDA 2  /* CUDA failure (CheckCudaError -> GpuMemoryException) */
#define ORX_EINTERNAL 3

/* AsrTextConfig, include/model/asr_text_decoder.h:30-43. The head geometry is
 * fixed at Qwen3-ASR-1.7B (2048 / 16 q / 8 kv / 128 / 6144) and checked. */
typedef struct orx_config {
  int hidden_size;
  int num_layers;
  int num_q_heads;
  int num_kv_heads;
  int head_dim;
  int intermediate_size;
  int vocab_size;
  float rms_norm_eps;
  float rope_theta;
  int max_seq_len;
  int profile;
  int cuda_graph_enabled;
} orx_config;

typedef struct orx_decoder orx_decoder;

const char* orx_last_error(void);
int orx_version(void);
/* Fills `cfg` with the AsrTextConfig defaults. */
void orx_config_default(orx_config* cfg);

/* AsrTextDecoder::AsrTextDecoder (asr_text_decoder.h:47); allocates weights,
 * the paged KV pool for max_seq_len positions and all step buffers on the
 * current device. */
int orx_decoder_create(const orx_config* cfg, orx_decoder** out);
void orx_decoder_destroy(orx_decoder* d);

/* AsrTextDecoder::LoadWeights (asr_text_decoder.cu:251-336), one tensor at a
 * time by its checkpoint name (thinker.model.*). dtype 0 = fp32, 1 = bf16 bits;
 * on_device = 1 if `data` is a device pointer. */
int orx_decoder_set_tensor(orx_decoder* d, const char* name, const void* data, int dtype,
                           size_t numel, int on_device);
/* Loads a sharded safetensors checkpoint directory (model.safetensors.index.json
 * or model.safetensors), as io::ShardedSafeTensors feeds LoadWeights
 * (src/io/sharded_safetensor.cc). */
int orx_decoder_load_safetensors(orx_decoder* d, const char* model_dir);
/* Seeded synthetic weights generated on the device (no reference counterpart:
 * stands in for a checkpoint on machines without one). */
int orx_decoder_init_synthetic(orx_decoder* d, int seed);
int orx_decoder_weights_complete(const orx_decoder* d, int* complete);

/* ResetCache / TruncateCache / cache_len (asr_text_decoder.h:51,73,76). */
int orx_decoder_reset_cache(orx_decoder* d);
int orx_decoder_truncate_cache(orx_decoder* d, int len);
int orx_decoder_cache_len(const orx_decoder* d, int* out);
/* Embed (asr_text_decoder.cu:340-346): bf16 row -> fp32 `out[hidden]` (host). */
int orx_decoder_embed(const orx_decoder* d, int token_id, float* out);

/* PrefillAt / Prefill (asr_text_decoder.cu:585-617): host embeds [T, hidden]
 * appended at pos0; logits of the last row stay on the device; synchronizes. */
int orx_decoder_prefill_at(orx_decoder* d, const float* embeds, int T, int pos0, void* stream);
/* Same with device-resident embeds; asynchronous on `stream`. */
int orx_decoder_prefill_at_device(orx_decoder* d, const float* d_embeds, int T, int pos0,
                                  void* stream);
/* DecodeStep (asr_text_decoder.cu:619-634): one host embedding at `pos`. */
int orx_decoder_decode_step(orx_decoder* d, const float* embed, int pos, void* stream);
/* DecodeStepDevice (asr_text_decoder.cu:655-671): token id read on the device. */
int orx_decoder_decode_step_device(orx_decoder* d, const int* d_token, int pos, void* stream);
/* Argmax / ArgmaxToDevice / ReadTokenId (asr_text_decoder.cu:636-653). */
int orx_decoder_argmax(orx_decoder* d, int ban0, int ban1, void* stream, int* out);
int orx_decoder_argmax_to_device(orx_decoder* d, int* d_out, int ban0, int ban1, void* stream);
int orx_decoder_read_token_id(const orx_decoder* d, const int* d_token, void* stream, int* out);
/* DecodeGreedy (asr_text_decoder.cu:698-889). `out_tokens` holds max_new ints;
 * *n_out receives the number of emitted tokens (EOS excluded). */
int orx_decoder_decode_greedy(orx_decoder* d, int start_pos, int max_new, int eos0, int eos1,
                              int ban_steps, int batch, void* stream, int* out_tokens, int* n_out);
/* CopyLogits (asr_text_decoder.cu:891-899): `out[vocab]` on the host. */
int orx_decoder_copy_logits(const orx_decoder* d, float* out);
/* Device pointer of the logits buffer (valid until destroy). */
int orx_decoder_logits_device(const orx_decoder* d, const float** out);
/* Device error word written by bounded waits (0 = none). */
int orx_decoder_device_error(const orx_decoder* d, int* out);

/* ---- Continuous batching (no single reference counterpart: replaces one
 * AsrTextDecoder per session, src/model/asr_text_decoder.cu:309-318, and the
 * per-session worker threads of src/pipeline/asr_worker.cc:270-416). Many
 * sessions share one paged KV pool (16-token pages) and the weights of an
 * existing decoder (`weights`, which must outlive the batch). */
typedef struct orx_batch orx_batch;
int orx_batch_create(orx_decoder* weights, int max_sessions, int max_batch, int pool_pages,
                     int max_pages_per_session, orx_batch** out);
void orx_batch_destroy(orx_batch* b);
/* New empty session (ORX_EINVAL when every slot is in use). */
int orx_batch_session_create(orx_batch* b, int* sid);
/* Ends a session and returns its pages to the pool. */
int orx_batch_session_free(orx_batch* b, int sid);
/* cache_len / TruncateCache per session (asr_text_decoder.h:73-76); truncation
 * returns whole pages beyond the new length to the pool. */
int orx_batch_cache_len(const orx_batch* b, int sid, int* out);
int orx_batch_truncate(orx_batch* b, int sid, int len);
int orx_batch_free_pages(const orx_batch* b, int* out);
/* PrefillAt for n sessions at once: lens[i] host embedding rows (concatenated
 * [sum lens, 2048] fp32) appended at each session's cache end; leaves each
 * session's next greedy token on the device. ORX_EINVAL and nothing changed
 * when the page pool cannot hold the rows (the join is rejected). */
int orx_batch_prefill(orx_batch* b, const int* sids, const int* lens, int n,
                      const float* embeds, void* stream);
/* One greedy decode token for each of the n sessions (ragged lengths) in one
 * batched step; tokens_out (host, n ints, may be NULL) receives them. */
int orx_batch_step(orx_batch* b, const int* sids, int n, int* tokens_out, void* stream);
int orx_batch_device_error(const orx_batch* b, int* out);
/* Ban window of DecodeGreedy (asr_text_decoder.cu:698-857) per session: the
 * session's next `steps` argmaxes (the one closing a prefill, then one per
 * step) exclude token ids ban0 and ban1 (-1: none). Ordered on `stream`. */
int orx_batch_set_ban(orx_batch* b, int sid, int ban0, int ban1, int steps, void* stream);
/* Each listed session's pending greedy token (produced by its last prefill or
 * step, fed by its next step), to host out[n]. Waits for `stream`. */
int orx_batch_next_tokens(orx_batch* b, const int* sids, int n, int* out, void* stream);

/* ---- fp32 single decoder layer (correctness configuration; no reference GPU
 * counterpart: the reference checks this layer in fp32 on its CPU oracle).
 * One Qwen3-1.7B-shaped layer with fp32 weights, activations and KV cache and
 * no bf16 rounding; rows are processed causally, each appending its K/V.
 * Tensor names are layer-relative ("self_attn.q_proj", "mlp.down_proj", ...,
 * as in thinker.model.layers.N.<name>.weight), fp32. */
typedef struct orx_layer32 orx_layer32;
/* Geometry from cfg must be the decoder's; uses max_seq_len, rms_norm_eps,
 * rope_theta (max_seq_len <= 51200). */
int orx_layer32_create(const orx_config* cfg, orx_layer32** out);
void orx_layer32_destroy(orx_layer32* l);
int orx_layer32_set_tensor(orx_layer32* l, const char* name, const float* data, size_t numel,
                           int on_device);
/* Seeded synthetic weights of decoder layer `layer`: the generator of
 * orx_decoder_init_synthetic without the bf16 rounding. */
int orx_layer32_init_synthetic(orx_layer32* l, int seed, int layer);
/* T rows [T, 2048] at positions pos0.. (pos0 <= cache length) -> layer
 * outputs [T, 2048]; host pointers, synchronous. */
int orx_layer32_forward(orx_layer32* l, const float* x, int T, int pos0, float* out, void* stream);
/* Same with device pointers, asynchronous on `stream`. */
int orx_layer32_forward_device(orx_layer32* l, const float* d_x, int T, int pos0, float* d_out,
                               void* stream);
int orx_layer32_cache_len(const orx_layer32* l, int* out);
int orx_layer32_truncate(orx_layer32* l, int len);

/* ---- The reference's free operators (device pointers, asynchronous on
 * `stream`, row-major; empty sizes are no-ops as in the reference). ---- */

/* asr_gemm::LinearPre (include/model/asr_gemm.h:36-38):
 * out[M,N] = act(in[M,K] @ W[N,K]^T + bias[N]) with bf16 operands and fp32
 * accumulation on the tcgen05 tensor cores. bias may be NULL; act 0 = none,
 * 1 = GELU (exact, erf), 2 = ReLU. Any M, N; K a multiple of 8 with 16-byte
 * aligned operands runs on the tensor cores, other K on a CUDA-core kernel. */
int orx_linear_pre(const uint16_t* in_bf16, const uint16_t* W_bf16, const float* bias,
                   float* out_f32, int M, int K, int N, int act, void* stream);
/* asr_gemm::Linear (asr_gemm.h:30-32): LinearPre after the fp32 -> bf16
 * (round-to-nearest-even) cast of `in` into a per-thread buffer that grows on
 * demand (as the reference's). */
int orx_linear(const float* in_f32, const uint16_t* W_bf16, const float* bias, float* out_f32,
               int M, int K, int N, int act, void* stream);
/* asr_gemm::F32ToBf16 / Bf16ToF32 (asr_gemm.h:24-26). */
int orx_f32_to_bf16(const float* in, uint16_t* out, long long n, void* stream);
int orx_bf16_to_f32(const uint16_t* in, float* out, long long n, void* stream);
/* asr_ops::RmsNorm (include/model/asr_ops.cuh:22-25): out = x * rsqrt(mean(x^2)
 * + eps) * weight per row; in place allowed. */
int orx_rms_norm(const float* x, const float* weight, float* out, int rows, int dim, float eps,
                 void* stream);
/* asr_ops::RopeHalf (asr_ops.cuh:41-48) and asr_ops::RopeInterleaved
 * (asr_ops.cuh:27-34): rotary embedding in place over x [n_tokens, n_heads,
 * head_dim] at positions [n_tokens] (device ints); head_dim even. */
int orx_rope_half(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                  float theta_base, void* stream);
int orx_rope_interleaved(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                         float theta_base, void* stream);
/* asr_ops::SwiGLU (asr_ops.cuh:36-39): out = gate / (1 + exp(-gate)) * up. */
int orx_swiglu(const float* gate, const float* up, float* out, long long n, void* stream);
/* asr_ops::GqaAttention (asr_ops.cuh:50-56): q [T,Hq,D], k/v [T,Hkv,D] ->
 * out [T,Hq,D], fp32, online softmax; Hq a multiple of Hkv, D <= 1024. */
int orx_gqa_attention(const float* q, const float* k, const float* v, float* out, int T, int Hq,
                      int Hkv, int head_dim, float scale, int causal, void* stream);
/* asr_ops::ArgmaxBanned (asr_ops.cuh:58-62): index of the largest of n fp32
 * logits, skipping ban0 / ban1 (-1 = none), into the device int d_out; exact
 * ties, NaN and values <= -1e30 are handled as the reference kernel does.
 * Uses no scratch memory (one CTA). */
int orx_argmax_banned(const float* logits, int n, int ban0, int ban1, int* d_out, void* stream);

/* Diagnostic (no reference counterpart): average device ms per launch of each
 * decode kernel class, ms[6] = {qkv GEMV, attention, o GEMV, gate/up GEMV,
 * down GEMV, lm_head GEMV}, each timed over `iters` back-to-back launches with
 * CUDA events on `stream`. Clobbers the step buffers and the KV entry at the
 * current position; call it only between requests. */
int orx_decoder_profile_kernels(orx_decoder* d, int iters, void* stream, float* ms);

/* Diagnostic (no reference counterpart): runs `steps` decode steps from the
 * current cache end, feeding back its own greedy tokens, and writes per kernel
 * launch {first block start, last block past its dependency wait, last block
 * end} in GPU global-timer nanoseconds to out[steps * L * 3], L = 5 * layers + 1
 * (returned in *launches_per_step). Advances cache_len by `steps`. */
int orx_decoder_trace_decode(orx_decoder* d, int steps, void* stream, unsigned long long* out,
                             int* launches_per_step);
/* Diagnostic (no reference counterpart), persistent decode kernel only: like
 * trace_decode, but per phase and per CTA: out[(k * grid + cta) * 2 + {0, 1}]
 * = {inputs of phase k ready, phase k done} for k < steps * L, global-timer ns;
 * *grid receives the CTA count. ORX_EINVAL when the persistent kernel is off. */
int orx_decoder_trace_ctas(orx_decoder* d, int steps, void* stream, unsigned long long* out,
                           size_t out_len, int* grid);

/* Allocation-free banned argmax (no counterpart in the reference; the same
 * index as orx_decoder_argmax_to_device and asr_ops::ArgmaxBanned on the same
 * logits, exact ties included).
 * For callers that cannot allocate device memory: code inside a stream capture
 * it does not own, real-time threads that must not take the driver's
 * allocation locks, or processes whose device memory is reserved by another
 * allocator. Writes the index of the largest of `n` fp32 device logits,
 * skipping ban0/ban1 (-1 = none; ties resolved as asr_ops::ArgmaxBanned does), to the device
 * int `d_out`, asynchronously on `stream`. Its only scratch is a fixed 8,200-byte
 * array compiled into the library (held by every GPU that loads it until exit),
 * so n is limited to 8,388,608; larger n is rejected with ORX_EINVAL. The first
 * call on each device (with that device current) looks up the array's address;
 * make that first call before any stream capture. All calls on one device share
 * the array and it keeps the last call's contents: calls that overlap on the
 * GPU (e.g. on concurrent streams) race and must be serialized by the caller.
 * Allocates nothing. */
int orx_argmax_banned_noalloc(const float* d_logits, int n, int ban0, int ban1, int* d_out,
                              void* stream);

/* ---- Batched speech detector (the Silero-shaped model of the reference's
 * GpuVad, src/pipeline/gpu_vad.cu, batched over streams instead of over one
 * stream's windows). ---- */
typedef struct orx_vad orx_vad;
/* GpuVad::GpuVad (include/pipeline/gpu_vad.h:40): `streams` independent
 * streams, LSTM state and 64-sample context zeroed, on the current device. */
int orx_vad_create(int streams, orx_vad** out);
void orx_vad_destroy(orx_vad* v);
/* GpuVad::LoadWeights (gpu_vad.cu:242-271), one fp32 host tensor at a time by
 * its checkpoint name ("stft.forward_basis_buffer", "encoder.{0..3}.reparam_conv.
 * {weight,bias}", "decoder.rnn.{weight,bias}_{ih,hh}", "decoder.decoder.2.{weight,bias}"). */
int orx_vad_set_tensor(orx_vad* v, const char* name, const float* data, size_t numel);
/* Seeded synthetic weights (no reference counterpart; test and bench data). */
int orx_vad_init_synthetic(orx_vad* v, int seed);
/* GpuVad::Reset (gpu_vad.cu:471-483): every stream's LSTM state and context. */
int orx_vad_reset(orx_vad* v);
/* GpuVad::RunBatch (gpu_vad.cu:320-368) for all streams at once: pcm
 * [streams][steps * 512] fp32 -> speech probabilities probs [streams][steps];
 * both on the device (on_device = 1, asynchronous on `stream`) or both on the
 * host (synchronous). State carries over to the next call. */
int orx_vad_run(orx_vad* v, const float* pcm, int steps, float* probs, int on_device,
                void* stream);

/* ---- Audio tower (the Qwen3-ASR encoder that produces the decoder's audio
 * rows; AsrAudioTower, include/model/asr_audio_tower.h:52-128), batched over
 * utterances. ---- */
typedef struct orx_tower orx_tower;
/* AsrAudioTower::AsrAudioTower (asr_audio_tower.h:54) with
 * AsrAudioConfig::encoder_layers = `layers` and windowed_attention =
 * `windowed` (other fields at their defaults: 128 mel bins, d_model 1024,
 * 16 heads, ffn 4096, downsample 480, output 2048, 100-frame chunks). */
int orx_tower_create(int layers, int windowed, orx_tower** out);
void orx_tower_destroy(orx_tower* t);
/* One host tensor by checkpoint name (thinker.audio_tower.*); dtype 0 = fp32,
 * 1 = bf16 bits. Matrices are held in bf16, vectors in fp32 (as
 * AsrAudioTower::LoadWeights, asr_audio_tower.cu:318-361). */
int orx_tower_set_tensor(orx_tower* t, const char* name, const void* data, int dtype,
                         size_t numel);
/* AsrAudioTower::LoadWeights(ShardedSafeTensors) from a model directory. */
int orx_tower_load_safetensors(orx_tower* t, const char* dir);
/* Seeded synthetic weights (no reference counterpart; test and bench data). */
int orx_tower_init_synthetic(orx_tower* t, int seed);
int orx_tower_weights_complete(const orx_tower* t, int* complete);
/* AsrAudioTower::OutputLength (asr_audio_tower.cu:279-283). */
int orx_tower_output_length(int n_frames);
/* AsrAudioTower::Forward (asr_audio_tower.h:77-78): mel [128, n_frames] fp32
 * (host) -> out [OutputLength(n_frames), 2048] fp32 (host); *out_tokens gets
 * the row count. Synchronous on `stream`. */
int orx_tower_forward(orx_tower* t, const float* mel, int n_frames, float* out, int* out_tokens,
                      void* stream);
/* Many utterances in one call (no reference counterpart: the batched form).
 * d_mel: the n utterances' [128, frames[u]] blocks back to back (device);
 * frames: host array; d_out: [sum OutputLength(frames[u]), 2048] (device),
 * utterance u's rows after those of u - 1. Attention never crosses
 * utterances. Asynchronous on `stream`; *out_rows gets the total rows. */
int orx_tower_forward_batch(orx_tower* t, const float* d_mel, const int* frames, int n,
                            float* d_out, int* out_rows, void* stream);

/* ---- Streaming Sortformer diarizer network (ConformerPreEncode,
 * ConformerLayer x 17, SortformerDecoder: include/model/conformer_preencode.h,
 * conformer_layer.h, sortformer_decoder.h), fp32 model. ---- */
typedef struct orx_sf orx_sf;
/* `conf_layers` FastConformer layers (17 in the reference) and `dec_layers`
 * transformer layers (18), d 512 / 192, 4 speakers. */
int orx_sf_create(int conf_layers, int dec_layers, orx_sf** out);
void orx_sf_destroy(orx_sf* s);
/* One fp32 host tensor by checkpoint name (encoder.pre_encode.*,
 * encoder.layers.N.*, sortformer_modules.*, transformer_encoder.layers.N.*),
 * as the reference's LoadWeights read them. */
int orx_sf_set_tensor(orx_sf* s, const char* name, const float* data, size_t numel);
/* Every known tensor of one F32 safetensors file (SafeTensorReader). */
int orx_sf_load_safetensors(orx_sf* s, const char* path);
/* Seeded synthetic weights (no reference counterpart; test and bench data). */
int orx_sf_init_synthetic(orx_sf* s, int seed);
int orx_sf_weights_complete(const orx_sf* s, int* complete);
/* ConformerPreEncode::Forward (conformer_preencode.cu:196-279): mel
 * [128, n_frames] freq-major -> out [T2, 512], T2 = three stride-2 stages of
 * n_frames; *valid_out = the same of `valid`. on_device: pointers are device
 * memory and the call is asynchronous on `stream`; else host, synchronous. */
int orx_sf_pre_encode(orx_sf* s, const float* mel, int n_frames, int valid, float* out, int* T_out,
                      int* valid_out, int on_device, void* stream);
/* SortformerDiarizer::ForwardEncoderDecoder (streaming_sortformer.cc:391-418):
 * emb [T, 512] -> per-frame speaker probabilities preds [T, 4], rows >= valid
 * zero. */
int orx_sf_forward(orx_sf* s, const float* emb, int T, int valid, float* preds, int on_device,
                   void* stream);
/* One streaming step (StreamMelChunk's network part, streaming_sortformer.cc
 * :468-537): pre-encode the chunk's mel, put the n_cache speaker-cache + FIFO
 * rows [n_cache, 512] in front, run the encoder and decoder: preds [T, 4]
 * with T = n_cache + T2 (*T_out), valid rows n_cache + valid2 (*valid_out). */
int orx_sf_step(orx_sf* s, const float* mel, int n_frames, int valid, const float* cache,
                int n_cache, float* preds, int* T_out, int* valid_out, int on_device, void* stream);

/* Seeded synthetic fp32 data on the device, bit-exact with oracle/synth.py
 * (test and benchmark inputs; no reference counterpart). */
int orx_synth_f32(float* d_out, long long n, int seed, int tensor_id, double std, float mean,
                  int round_bf16, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ORX_H_ */
