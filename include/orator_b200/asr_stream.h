// Multi-session streaming front door (C++), the decoder side of the
// reference's Qwen3Asr::StreamReset / StreamChunk / StreamDecodeStep
// (src/model/qwen3_asr.cc:269-304, 307-407, 503-557) for many sessions that
// share one AsrSessionPool:
//   Open          prefix <|im_start|>system\n{system}<|im_end|>\n
//                 <|im_start|>user\n<|audio_start|> at position 0; the
//                 checkpoint is its length
//   AppendAudio   encoder rows after the checkpoint, which moves past them
//   Decode        per session: suffix <|audio_end|><|im_end|>\n<|im_start|>
//                 assistant\n{language}<asr_text>{committed} after the
//                 checkpoint, greedy decode with DecodeGreedy's rules (EOS
//                 banned for the first ban_steps argmaxes; stop at EOS or six
//                 equal tokens; at most max_new), truncate to the checkpoint.
//                 All requested sessions step together (one batched step per
//                 token).
// Token ids in, token ids out: the tokenizer and the text rollback stay with
// the caller, as in the reference.
#pragma once

#include <map>
#include <vector>

#include "orator_b200/asr_text_decoder.h"

namespace orator {
namespace model {

struct AsrStreamTokens {
  // Special ids of Qwen3-ASR (include/model/qwen3_asr.h:193-203).
  static constexpr int kImStart = 151644, kImEnd = 151645, kEndOfText = 151643;
  static constexpr int kAudioStart = 151669, kAudioEnd = 151670, kAsrText = 151704;
  static constexpr int kSystem = 8948, kUser = 872, kAssistant = 77091, kNewline = 198;
};

class AsrStreamPool {
 public:
  struct Request {
    std::vector<int> language;   // token ids of "language X" (may be empty)
    std::vector<int> committed;  // token ids of the committed prefix text
  };

  AsrStreamPool(const AsrTextDecoder& weights, AsrSessionPool& pool, int max_new = 32,
                int ban_steps = 3, int eos0 = AsrStreamTokens::kImEnd,
                int eos1 = AsrStreamTokens::kEndOfText);

  int Open(const std::vector<int>& system_ids, cudaStream_t stream = 0);
  void Close(int session);
  // rows[i]: T_i x hidden encoder rows of session sessions[i] (host).
  void AppendAudio(const std::vector<int>& sessions, const std::vector<const float*>& rows,
                   const std::vector<int>& lens, cudaStream_t stream = 0);
  std::map<int, std::vector<int>> Decode(const std::map<int, Request>& requests,
                                         cudaStream_t stream = 0);
  int checkpoint(int session) const { return ckpt_.at(session); }

  static std::vector<int> PrefixIds(const std::vector<int>& system_ids);
  static std::vector<int> SuffixIds(const Request& r);

 private:
  std::vector<float> EmbedRows(const std::vector<int>& ids) const;

  const AsrTextDecoder& w_;
  AsrSessionPool& pool_;
  int max_new_, ban_steps_, eos0_, eos1_;
  std::map<int, int> ckpt_;
};

}  // namespace model
}  // namespace orator
