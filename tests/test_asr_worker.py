"""The session scheduler (include/orator_b200/asr_worker.h: AsrWorker,
VadEvidenceStore, StreamBatcher), compiled with g++ against the built library
and driven by a scripted recognizer, on the CPU.

AsrWorker cases follow the reference's own worker test
(test/unit/pipeline/test_asr_worker.cc): stable text ids across finals,
partial de-duplication, full-context finals, retraction of an empty final,
silence skipped from VAD evidence, the VAD gate's reset positions, feed
quanta, exact fed samples and final bounds (and their independence from the
order in which VAD evidence is published), speech resuming inside the
trailing interval, the long-gap lead, the terminal drain; plus the
segment_sec and max_audio_tokens caps. StreamBatcher: eight worker threads
sharing one batched decoder get their own streams' text back and their decoder
calls coalesce into multi-stream batches."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "orator_b200")
CUDA_INC = "/usr/local/cuda/include"

PROGRAM = r"""
#include <algorithm>
#include <cstdio>
#include <numeric>
#include <string>
#include <thread>
#include <vector>
#include "orator_b200/asr_worker.h"
using namespace orator;
using pipeline::AsrWorker;
using pipeline::VadEvidenceStore;

static int fails = 0;
#define EXPECT(c) do { if (!(c)) { std::printf("FAIL line %d: %s\n", __LINE__, #c); ++fails; } } while (0)

// Scripted recognizer: returns the next scripted text per chunk (or keeps
// the last), records what it was given.
struct Script : core::IStreamAsr {
  std::vector<std::string> outs; size_t at = 0; std::string cur, final_text;
  std::vector<long> resets; std::vector<int> chunks; std::vector<float> fed, final_pcm;
  int finals = 0, tokens = 1;
  void Reset() override {}
  void StreamReset(long b) override { resets.push_back(b); cur = "speech"; }
  std::string StreamChunk(const float* p, int n, cudaStream_t) override {
    chunks.push_back(n); fed.insert(fed.end(), p, p + n);
    if (at < outs.size()) cur = outs[at++];
    return cur;
  }
  std::string StreamFinalize(cudaStream_t) override { return cur; }
  std::string TranscribeFinal(const float* p, int n, cudaStream_t) override {
    final_pcm.assign(p, p + n); ++finals; return final_text;
  }
  int stream_audio_tokens() const override { return tokens; }
};

struct Final { long id; double s, e; std::string t;
  bool operator==(const Final& o) const { return id == o.id && s == o.s && e == o.e && t == o.t; } };
struct Run { std::vector<long> resets; std::vector<int> chunks; std::vector<float> fed;
             std::vector<std::string> events; std::vector<Final> finals; size_t early_events = 0; };

static AsrWorker::Params gate_params(double trail) {
  AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = true;
  p.asr_vad_lead_ms = 100; p.asr_vad_gate_chunk_ms = 100; p.asr_vad_trail_sec = trail;
  p.asr_vad_min_overlap_sec = 0.01; return p;
}

// Speech [0.2, 0.4) and [gap_start, gap_end), VAD decided to 1.0 s, published
// in one of three orders relative to the audio.
static Run gate_run(int order, double s2, double e2) {
  Script asr; VadEvidenceStore ev; Run r;
  AsrWorker w(&asr, gate_params(0.1), [&](const std::string& e) { r.events.push_back(e); },
              core::TimeBase(100), 0, &ev);
  w.set_text_sink([&](long id, double s, double e, const std::string& t, bool fin) {
    if (fin) r.finals.push_back({id, s, e, t}); });
  std::vector<float> a(100); std::iota(a.begin(), a.end(), 0.0f);
  auto publish = [&] { ev.DepositVad({0.2, 0.4}); ev.DepositVad({s2, e2});
                       ev.UpdateVadState(false, 1.0); ev.AdvanceVadHorizon(1.0); };
  if (order == 0) { publish(); w.ProcessSpan(a.data(), 100); }
  else if (order == 1) { w.ProcessSpan(a.data(), 10); r.early_events = r.events.size(); publish();
                         w.ProcessSpan(a.data() + 10, 90); }
  else { ev.UpdateVadState(true, 0.8, 0.2, 0.45); w.ProcessSpan(a.data(), 50); publish();
         w.ProcessSpan(a.data() + 50, 50); }
  w.Finalize();
  r.resets = asr.resets; r.chunks = asr.chunks; r.fed = asr.fed; return r;
}

int main() {
  // text ids are stable across two finals, in events and in the sink
  {
    Script asr; AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = false;
    std::vector<std::string> ev; std::vector<long> ids;
    AsrWorker w(&asr, p, [&](const std::string& e) { ev.push_back(e); }, core::TimeBase(100));
    w.set_text_sink([&](long id, double, double, const std::string&, bool f) { if (f) ids.push_back(id); });
    std::vector<float> a(10, 0.25f);
    w.ProcessSpan(a.data(), 10); w.Finalize(); w.ProcessSpan(a.data(), 10); w.Finalize();
    EXPECT(ids == std::vector<long>({0, 1}));
    int f0 = 0, f1 = 0;
    for (auto& e : ev) if (e.find("\"type\":\"asr\"") != std::string::npos) {
      f0 += e.find("\"text_id\":0") != std::string::npos; f1 += e.find("\"text_id\":1") != std::string::npos; }
    EXPECT(f0 == 1 && f1 == 1);
  }
  // an unchanged partial is published once; changed ones each once, in order
  for (int changing = 0; changing < 2; ++changing) {
    Script asr; asr.outs = changing ? std::vector<std::string>{"first", "second"}
                                    : std::vector<std::string>{"speech", "speech"};
    AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = false;
    std::vector<std::string> ev; int typed = 0;
    AsrWorker w(&asr, p, [&](const std::string& e) { ev.push_back(e); }, core::TimeBase(100));
    w.set_text_sink([&](long, double, double, const std::string&, bool f) { if (!f) ++typed; });
    std::vector<float> a(20, 0.25f);
    w.ProcessSpan(a.data(), 10); w.ProcessSpan(a.data() + 10, 10); w.Finalize();
    std::vector<std::string> partial;
    for (auto& e : ev) if (e.find("asr_partial") != std::string::npos) partial.push_back(e);
    EXPECT(typed == (changing ? 2 : 1) && partial.size() == (changing ? 2u : 1u));
    if (changing && partial.size() == 2)
      EXPECT(partial[0].find("\"text\":\"first\"") != std::string::npos &&
             partial[1].find("\"text\":\"second\"") != std::string::npos);
  }
  // full-context final: one decode over exactly the admitted PCM replaces the live text
  {
    Script asr; asr.outs = {"provisional"}; asr.final_text = "full context";
    AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = false;
    p.final_full_context_decode = true;
    std::vector<Final> fin;
    AsrWorker w(&asr, p, [](const std::string&) {}, core::TimeBase(100));
    w.set_text_sink([&](long id, double s, double e, const std::string& t, bool f) { if (f) fin.push_back({id, s, e, t}); });
    std::vector<float> a(20); std::iota(a.begin(), a.end(), 0.0f);
    w.ProcessSpan(a.data(), 10); w.ProcessSpan(a.data() + 10, 10); w.Finalize();
    EXPECT(asr.finals == 1 && asr.final_pcm == a && fin.size() == 1 && fin[0].t == "full context");
  }
  // an empty full-context final retracts the live text and deposits nothing
  {
    Script asr; asr.outs = {"provisional"}; asr.final_text = "";
    AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = false;
    p.final_full_context_decode = true;
    std::vector<std::string> ev; int nf = 0;
    AsrWorker w(&asr, p, [&](const std::string& e) { ev.push_back(e); }, core::TimeBase(100));
    w.set_text_sink([&](long, double, double, const std::string&, bool f) { nf += f; });
    std::vector<float> a(10, 0.25f); w.ProcessSpan(a.data(), 10); w.Finalize();
    EXPECT(nf == 0 && std::any_of(ev.begin(), ev.end(), [](const std::string& e) {
      return e.find("\"type\":\"asr_retract\"") != std::string::npos; }));
  }
  // silence decided by VAD (horizon only, or horizon + silent state) is skipped
  for (int state = 0; state < 2; ++state) {
    Script asr; VadEvidenceStore ev; ev.AdvanceVadHorizon(1.0);
    if (state) ev.UpdateVadState(false, 1.0);
    AsrWorker::Params p = gate_params(1.5); p.asr_vad_min_overlap_sec = 0.12;
    std::vector<std::string> events; int nf = 0;
    AsrWorker w(&asr, p, [&](const std::string& e) { events.push_back(e); }, core::TimeBase(100), 0, &ev);
    w.set_text_sink([&](long, double, double, const std::string&, bool f) { nf += f; });
    std::vector<float> a(100, 0.0f); w.ProcessSpan(a.data(), 100); w.Finalize();
    EXPECT(w.processed_samples() == 100 && events.empty() && nf == 0 && asr.resets.empty() && asr.fed.empty());
  }
  // the gate: publication order of the VAD evidence does not change anything
  {
    Run a = gate_run(0, 0.45, 0.5), b = gate_run(1, 0.45, 0.5), c = gate_run(2, 0.45, 0.5);
    EXPECT(b.early_events == 0);
    EXPECT(a.resets == b.resets && a.resets == c.resets);
    EXPECT(a.chunks == b.chunks && a.chunks == c.chunks);
    EXPECT(a.fed == b.fed && a.fed == c.fed);
    EXPECT(a.events == b.events && a.events == c.events);
    EXPECT(a.finals == b.finals && a.finals == c.finals);
    EXPECT(a.resets == std::vector<long>{10});                    // onset 0.2 s minus the 0.1 s lead
    EXPECT(a.chunks == std::vector<int>({10, 10, 10, 5, 5}));     // quanta, then the kept gap
    EXPECT(a.fed.size() == 40 && a.fed.front() == 10.0f && a.fed.back() == 49.0f);
    EXPECT(a.finals.size() == 1 && a.finals[0].s == 0.1 && a.finals[0].e == 0.6);
  }
  {
    Run a = gate_run(0, 0.55, 0.7), b = gate_run(1, 0.55, 0.7);
    EXPECT(a.resets == std::vector<long>({10, 45}) && a.resets == b.resets);
    EXPECT(a.chunks == b.chunks && a.fed == b.fed && a.events == b.events && a.finals == b.finals);
  }
  // speech back within the trailing interval stays in one session; a long gap
  // closes it and the next session starts at its own lead
  {
    for (int longgap = 0; longgap < 2; ++longgap) {
      Script asr; VadEvidenceStore ev;
      ev.DepositVad({0.2, 0.4}); ev.DepositVad(longgap ? VadEvidenceStore::VadSeg{0.55, 0.7}
                                                      : VadEvidenceStore::VadSeg{0.45, 0.6});
      ev.AdvanceVadHorizon(1.0);
      std::vector<Final> fin;
      AsrWorker w(&asr, gate_params(0.1), [](const std::string&) {}, core::TimeBase(100), 0, &ev);
      w.set_text_sink([&](long id, double s, double e, const std::string& t, bool f) { if (f) fin.push_back({id, s, e, t}); });
      std::vector<float> a(100); std::iota(a.begin(), a.end(), 0.0f);
      w.ProcessSpan(a.data(), 100); w.Finalize();
      if (!longgap) {
        EXPECT(asr.resets == std::vector<long>{10});
        EXPECT(asr.fed == std::vector<float>(a.begin() + 10, a.begin() + 60));
        EXPECT(fin.size() == 1 && fin[0].s == 0.1 && fin[0].e == 0.7);
      } else {
        EXPECT(asr.resets == std::vector<long>({10, 45}));
        EXPECT(fin.size() == 2 && fin[0].s == 0.1 && fin[0].e == 0.5 && fin[1].s == 0.45 && fin[1].e == 0.8);
      }
    }
  }
  // terminal drain keeps only the trailing bound the audio has
  {
    Script asr; VadEvidenceStore ev; ev.DepositVad({0.8, 0.95}); ev.UpdateVadState(false, 1.0);
    ev.AdvanceVadHorizon(1.0);
    std::vector<Final> fin;
    AsrWorker w(&asr, gate_params(0.2), [](const std::string&) {}, core::TimeBase(100), 0, &ev);
    w.set_text_sink([&](long id, double s, double e, const std::string& t, bool f) { if (f) fin.push_back({id, s, e, t}); });
    std::vector<float> a(100); std::iota(a.begin(), a.end(), 0.0f);
    w.ProcessSpan(a.data(), 100); w.Finalize();
    EXPECT(asr.resets == std::vector<long>{70});
    EXPECT(asr.fed == std::vector<float>(a.begin() + 70, a.begin() + 95));
    EXPECT(fin.size() == 1 && fin[0].s == 0.7 && fin[0].e == 1.0);
  }
  // caps: segment_sec closes a segment after 0.3 s of audio; max_audio_tokens
  // closes it as soon as the decoder reports that many tokens
  {
    Script asr; AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.3; p.asr_vad_gate = false;
    std::vector<Final> fin;
    AsrWorker w(&asr, p, [](const std::string&) {}, core::TimeBase(100));
    w.set_text_sink([&](long id, double s, double e, const std::string& t, bool f) { if (f) fin.push_back({id, s, e, t}); });
    std::vector<float> a(10, 1.0f);
    for (int i = 0; i < 7; ++i) w.ProcessSpan(a.data(), 10);
    w.Finalize();
    EXPECT(asr.resets == std::vector<long>({0, 30, 60}));
    EXPECT(fin.size() == 3 && fin[0].e == 0.3 && fin[1].s == 0.3 && fin[2].e == 0.7);
  }
  {
    Script asr; asr.tokens = 0; AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0;
    p.asr_vad_gate = false; p.max_audio_tokens = 5;
    int nf = 0;
    AsrWorker w(&asr, p, [](const std::string&) {}, core::TimeBase(100));
    w.set_text_sink([&](long, double, double, const std::string&, bool f) { nf += f; });
    std::vector<float> a(10, 1.0f);
    w.ProcessSpan(a.data(), 10); w.ProcessSpan(a.data(), 10);
    EXPECT(nf == 0);
    asr.tokens = 5; w.ProcessSpan(a.data(), 10);
    EXPECT(nf == 1 && asr.resets.size() == 1);
  }
  // many streams, one batched decoder
  {
    const int S = 8;
    std::vector<int> calls(S, 0);
    pipeline::StreamBatcher::StreamOps ops;
    ops.audio_tokens = [](int) { return 0; };
    pipeline::StreamBatcher batcher(
        S,
        [&](const std::vector<pipeline::StreamBatcher::Request>& rq, std::vector<std::string>* out) {
          for (size_t i = 0; i < rq.size(); ++i) {
            const int s = rq[i].stream;
            (*out)[i] = rq[i].finalize ? "final" + std::to_string(s)
                                       : "s" + std::to_string(s) + ":" + std::to_string(++calls[s]) +
                                         ":" + std::to_string(static_cast<int>(rq[i].pcm[0]));
          }
        },
        ops, std::chrono::microseconds(200000));
    std::vector<std::vector<Final>> fins(S);
    std::vector<std::vector<std::string>> partials(S);
    std::vector<std::thread> th;
    for (int s = 0; s < S; ++s) th.emplace_back([&, s] {
      AsrWorker::Params p; p.sample_rate = 100; p.segment_sec = 0.0; p.asr_vad_gate = false;
      AsrWorker w(batcher.Stream(s), p, [](const std::string&) {}, core::TimeBase(100));
      w.set_text_sink([&, s](long id, double a0, double a1, const std::string& t, bool f) {
        if (f) fins[s].push_back({id, a0, a1, t}); else partials[s].push_back(t); });
      std::vector<float> pcm(10, static_cast<float>(s));
      for (int k = 0; k < 5; ++k) { batcher.Enter(s); w.ProcessSpan(pcm.data(), 10); batcher.Leave(s); }
      batcher.Enter(s); w.Finalize(); batcher.Leave(s);
    });
    for (auto& t : th) t.join();
    for (int s = 0; s < S; ++s) {
      EXPECT(partials[s].size() == 5 && partials[s].back() == "s" + std::to_string(s) + ":5:" + std::to_string(s));
      EXPECT(fins[s].size() == 1 && fins[s][0].t == "final" + std::to_string(s) && fins[s][0].e == 0.5);
    }
    auto sizes = batcher.batch_sizes();
    int total = 0, big = 0;
    for (int z : sizes) { total += z; big = std::max(big, z); }
    EXPECT(total == S * 6);
    EXPECT(big > 1);                 // calls of different streams shared a batch
    EXPECT(sizes.size() < static_cast<size_t>(S * 6));
  }
  std::printf("%s\n", fails ? "FAIL" : "OK");
  return fails;
}
"""


def test_asr_worker_cases(tmp_path):
    if shutil.which("g++") is None or not os.path.isdir(CUDA_INC):
        pytest.skip("g++ or CUDA headers not available")
    if not os.path.exists(os.path.join(LIB_DIR, "liborator_b200.so")):
        from orator_b200.build import build
        build()
    src = tmp_path / "w.cc"
    src.write_text(PROGRAM)
    exe = tmp_path / "w"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pthread", "-I",
                    os.path.join(ROOT, "include"), "-I", CUDA_INC, str(src), "-o", str(exe),
                    "-L", LIB_DIR, "-l:liborator_b200.so", f"-Wl,-rpath,{LIB_DIR}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
