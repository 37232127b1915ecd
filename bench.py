"""Benchmark of the Qwen3-ASR text-decoder hot path on B200.

Workload (config 2 of the benchmark set): the 28-layer Qwen3-ASR-1.7B-shaped decoder in
bf16 with seeded synthetic weights (seed 1); a 400-row prompt (375 audio rows
N(0,1) + 25 token embeddings) is prefilled, then one bench step greedily
decodes 128 tokens at batch 1 (KV length 401..528). Every step replays the
same positions (the cache is truncated back to 400 first).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun every rank decodes its own independent session on its own GPU
(no collective on the data path, weak scaling); `value` is the aggregate.
`--impl reference` times the reference's CPU path for this decoder -- the
oracle restatement in oracle/ (the reference runtime itself is CUDA-only) --
on the host cores.

`roofline.traffic` is DRAM bytes from an ncu capture (dram__bytes_read.sum +
dram__bytes_write.sum) of a 4-token decode_mk_kernel launch of this workload,
3.4924 GB per token, scaled to the 128-token launch (weights exceed L2, so
traffic grows in proportion to tokens).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_ROWS, AUDIO_ROWS, SEED = 400, 375, 1
NEW_TOKENS = 128
HIDDEN, LAYERS, VOCAB = 2048, 28, 151936
# bytes streamed per decode token: bf16 matrices (incl. tied lm_head) + fp32 norms
WEIGHT_BYTES = 3_440_902_144 + 495_616
KV_BYTES_PER_POS = 28 * 2 * 8 * 128 * 2
METRIC = "decode tokens/s (B=1, Qwen3-ASR-1.7B text decoder, bf16)"


WORKLOAD2 = ("config2: 28-layer Qwen3-ASR-1.7B decoder, 400-row prefill, "
             "greedy decode of 128 tokens at B=1 (KV 401..528)")
NCU_BYTES_PER_TOKEN = 3.4924e9  # DRAM bytes per decode token, from ncu


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


class ClockSampler:
    """nvidia-smi samples during the timed region (read-only queries)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v
                          and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def _splitmix(x):
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        z = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def prompt_token_ids(n):
    """25 prompt ids uniform in [0, vocab) from the seeded counter hash (tensor id 60001)."""
    base = (np.uint64(SEED) << np.uint64(52)) | (np.uint64(60001) << np.uint64(36))
    h = _splitmix(base | np.arange(n, dtype=np.uint64))
    return ((h >> np.uint64(11)) % np.uint64(VOCAB)).astype(np.int32)


def build_prompt_gpu(dec, torch):
    from orator_b200 import synth_f32
    buf = torch.empty(AUDIO_ROWS * HIDDEN, dtype=torch.float32, device="cuda")
    synth_f32(buf.data_ptr(), buf.numel(), SEED, 60000, 1.0)
    torch.cuda.synchronize()
    audio = buf.cpu().numpy().reshape(AUDIO_ROWS, HIDDEN)
    toks = prompt_token_ids(PROMPT_ROWS - AUDIO_ROWS)
    emb = np.stack([dec.Embed(int(t)) for t in toks])
    # the prompt rows live in pinned host memory (the e2e leg copies them in)
    pinned = torch.empty((PROMPT_ROWS, HIDDEN), dtype=torch.float32, pin_memory=True)
    pinned.copy_(torch.from_numpy(np.concatenate([audio, emb], 0).astype(np.float32)))
    return pinned.numpy()


def cpu_oracle_rate(sample_tokens: int, warm: int = 1, reps: int = 1):
    """Times the CPU oracle (the restatement of the reference decoder) decoding
    `sample_tokens` greedy tokens at positions 400.. after a 400-row prefill."""
    import torch
    from oracle import decoder_oracle as D, synth
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = D.Config(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=PROMPT_ROWS + 64)
    o = D.OracleDecoder.synthetic(cfg, SEED)
    audio = synth.audio_rows(SEED, AUDIO_ROWS, HIDDEN)
    emb = np.concatenate([audio, o.embed.numpy()[prompt_token_ids(PROMPT_ROWS - AUDIO_ROWS)]], 0)
    o.prefill_at(emb, 0)
    logits0 = o.logits.copy()
    times = []
    for r in range(warm + reps):
        o.truncate(PROMPT_ROWS)
        o.logits = logits0.copy()
        t0 = time.perf_counter()
        o.decode_greedy(PROMPT_ROWS, sample_tokens, -1, -1, ban_steps=0, batch=sample_tokens)
        dt = time.perf_counter() - t0
        if r >= warm:
            times.append(dt)
    return sample_tokens / statistics.median(times), threads, times


def reference_gpu_rate(prompt, reps: int = 3):
    """The reference's own CUDA decoder on this GPU, for the same workload:
    the unmodified AsrTextDecoder compiled from its sources into
    oracle/_ref/libref_asr.so (oracle/build_ref.sh), loaded from a checkpoint
    with the same seeded weights, prefilled with the same 400 rows, then
    DecodeGreedy(400, 128 tokens, no EOS, batch 128) through its CUDA-graph
    loop (its fastest path), timed with CUDA events around the call."""
    import ctypes as C
    import shutil
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libref_asr.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref/libref_asr.so not built (oracle/build_ref.sh)"}
    import torch
    from oracle import st_writer, synth
    from orator_b200 import synth_f32

    def gen(seed, tid, shape, is_norm):
        n = int(np.prod(shape))
        buf = torch.empty(n, dtype=torch.float32, device="cuda")
        synth_f32(buf.data_ptr(), n, seed, tid, synth.NORM_STD if is_norm else synth.MATRIX_STD,
                  1.0 if is_norm else 0.0, True)
        return (buf.view(torch.int32) >> 16).to(torch.int16).cpu().numpy().view(np.uint16).reshape(shape)

    L = C.CDLL(lib_path)
    L.ref_create_graphs.restype = C.c_void_p
    L.ref_create_graphs.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int]
    L.ref_last_error.restype = C.c_char_p
    d = tempfile.mkdtemp(prefix="ref_ckpt_")
    try:
        st_writer.write_synthetic_model(d, SEED, LAYERS, VOCAB, shards=4, gen=gen)
        h = L.ref_create_graphs(d.encode(), LAYERS, VOCAB, 2048)
        if not h:
            return {"unavailable": "reference decoder failed to load: " + L.ref_last_error().decode()}
        h = C.c_void_p(h)
        x = np.ascontiguousarray(prompt, np.float32)
        assert L.ref_prefill_at(h, x.ctypes.data_as(C.c_void_p), PROMPT_ROWS, 0) == 0
        ms, n = C.c_float(), C.c_int()
        times = []
        for r in range(reps + 1):
            L.ref_truncate(h, PROMPT_ROWS)
            rc = L.ref_time_greedy(h, PROMPT_ROWS, NEW_TOKENS, NEW_TOKENS, C.byref(ms), C.byref(n))
            if rc != 0 or n.value != NEW_TOKENS:
                return {"unavailable": f"reference DecodeGreedy failed (rc {rc}, {n.value} tokens)"}
            if r:
                times.append(ms.value)
        L.ref_destroy(h)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    t = statistics.median(times)
    return {"value": NEW_TOKENS / (t * 1e-3), "unit": "tokens/s", "ms_per_step": t,
            "workload": WORKLOAD2,
            "note": "unmodified reference AsrTextDecoder (oracle/_ref) on this GPU, same weights "
                    "and prompt, DecodeGreedy with its CUDA-graph loop, median of "
                    f"{reps} after 1 warm-up"}


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    rate, threads, times = cpu_oracle_rate(args.cpu_sample, warm=1, reps=max(1, args.steps))
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": max(1, args.steps), "warmup": 1,
            "ms_per_step": 1e3 * statistics.median(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-rounded operands)",
            "data": "synthetic (seeded random-init weights, seeded N(0,1) audio rows)",
            "config": {"workload": WORKLOAD2, "global_batch": 1,
                       "parallelism": "host cores (rank 0 only)",
                       "sample": f"{args.cpu_sample} greedy tokens at KV 401..{400 + args.cpu_sample} per step",
                       "l2": "n/a (CPU)"},
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{args.cpu_sample} decode tokens after a 400-row prefill"},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ragged(dec, torch, world, dist, rank=0, strong=False, steps=256):
    """Config 3 of the benchmark set: 64 concurrent sessions, initial KV lengths
    U[128, 2048] (seed 2), 16-token pages; every 16 steps 8 sessions (drawn
    with the same generator) leave and 8 join with a 400-row prefill; 256 steps.
    weak: every GPU runs its own 64 sessions. strong: the 64 sessions are
    sharded over the GPUs by SessionRouter (least total KV length with room),
    joins included; every rank draws the same generator, so all agree on the
    placement without messages. Returns decode tokens / wall time including
    the joins' prefills (device time, max over ranks)."""
    from orator_b200 import BatchDecoder, synth_f32
    from orator_b200.router import SessionRouter
    rng = np.random.default_rng(2)
    B, STEPS, PAGE = 64, steps, 16
    init = rng.integers(128, 2049, B)
    max_pages = (2048 + STEPS + 400 + PAGE) // PAGE + 1
    pool = (B + 8) * max_pages
    bd = BatchDecoder(dec, max_sessions=B + 8, max_batch=B, pool_pages=pool,
                      max_pages_per_session=max_pages)
    router = SessionRouter(world if strong else 1, pool, PAGE)
    me = rank if strong else 0
    rows_buf = torch.empty(2048 * HIDDEN, dtype=torch.float32, device="cuda")

    def embeds(n, tid):
        synth_f32(rows_buf.data_ptr(), n * HIDDEN, SEED, tid, 1.0)
        torch.cuda.synchronize()
        return rows_buf[: n * HIDDEN].cpu().numpy().reshape(n, HIDDEN)

    gids = list(range(B))            # global session ids, in draw order
    local = {}                       # global id -> this rank's BatchDecoder session
    next_gid = B
    for i in range(B):  # initial histories (untimed)
        if router.place(i, int(init[i]), STEPS) == me:
            sid = bd.create_session()
            bd.prefill([sid], [embeds(int(init[i]), 61000 + i)])
            local[i] = sid
    joins = [embeds(PROMPT_ROWS, 62000 + j) for j in range(8)]
    # the join rows sit in pinned host memory, as an encoder's output would
    joins_pinned = torch.empty((8 * PROMPT_ROWS, HIDDEN), dtype=torch.float32, pin_memory=True)
    joins_pinned.copy_(torch.from_numpy(np.concatenate(joins, 0)))
    joins_cat = joins_pinned.numpy()
    # a rank that takes only some of the joins stages their rows here (pinned,
    # contiguous) so its prefill copy is asynchronous as in the full case
    stage = torch.empty((8 * PROMPT_ROWS, HIDDEN), dtype=torch.float32, pin_memory=True).numpy()

    # warm-up join (untimed): sizes the row buffers and split-K workspace for
    # an 8 x 400-row prefill, as the W warm-up steps do for the decode step
    warm = [bd.create_session() for _ in range(8)]
    bd.prefill(warm, joins_cat, lens=[PROMPT_ROWS] * 8)
    for w in warm:
        bd.free_session(w)

    def my_sids():
        return [local[g] for g in gids if g in local]

    for _ in range(3):  # warm-up: eager step, graph capture, replay (state is advanced)
        if my_sids():
            bd.step(my_sids())
        for g in gids:
            router.grow(g)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    sum_s = []
    s0 = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pre_ms = 0.0
    e0.record(s0)
    for step in range(STEPS):
        if step and step % 16 == 0:
            leave = rng.choice(len(gids), 8, replace=False)
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(s0)
            for k in sorted(leave, reverse=True):
                g = gids.pop(k)
                router.release(g)
                if g in local:
                    bd.free_session(local.pop(g))
            mine = []
            for j in range(8):
                g = next_gid
                next_gid += 1
                gids.append(g)
                if router.place(g, PROMPT_ROWS, STEPS) == me:
                    local[g] = bd.create_session()
                    mine.append((local[g], joins[j]))
            if len(mine) == 8:
                bd.prefill([m[0] for m in mine], joins_cat, lens=[PROMPT_ROWS] * 8)
            elif mine:
                for i, (_, rows_i) in enumerate(mine):
                    stage[i * PROMPT_ROWS:(i + 1) * PROMPT_ROWS] = rows_i
                bd.prefill([m[0] for m in mine], stage[:len(mine) * PROMPT_ROWS],
                           lens=[PROMPT_ROWS] * len(mine))
            p1.record(s0)
            p1.synchronize()
            pre_ms += p0.elapsed_time(p1)
        sum_s.append(sum(router.lens[g] + 1 for g in gids if g in local))
        if my_sids():
            bd.step(my_sids())
        for g in gids:
            router.grow(g)
    e1.record(s0)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    err = bd.device_error()
    bd.close()
    step_bytes = [WEIGHT_BYTES + KV_BYTES_PER_POS * x for x in sum_s]
    dec_ms = ms - pre_ms
    if dist:
        t = torch.tensor([ms, pre_ms, dec_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, pre_ms, dec_ms = t.tolist()
    tokens = B * STEPS * (1 if strong else world)
    hbm, kind = peaks()
    label = ("config3 strong: 64 ragged sessions sharded over the GPUs by least total KV length"
             if strong else "config3: 64 ragged sessions per GPU")
    return {"workload": label + ", KV U[128,2048] (seed 2), 8 leave + 8 join (400-row prefill) "
                                f"every 16 steps, {STEPS} steps",
            "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "scaling": "strong" if strong else "weak", "ms_total": ms, "ms_prefill_joins": pre_ms,
            "decode_only_tokens_per_s": tokens / (dec_ms / 1e3),
            "mean_sum_kv_rank": float(np.mean(sum_s)),
            "step_hbm_rank": {"bytes_per_step_mean": float(np.mean(step_bytes)),
                              "achieved_gbs": float(np.sum(step_bytes)) / (dec_ms * 1e-3) / 1e9,
                              "frac": float(np.sum(step_bytes)) / (dec_ms * 1e-3) / 1e9 / hbm},
            "device_error": err}


def run_config1(torch, hbm, cpu: bool):
    """Config 1: one fp32 decoder layer (seed 0), KV of 512 past positions built
    by the layer itself from 512 N(0,1) rows, then one decode row at position
    512, timed with CUDA events (truncate back to 512 between reps); the CPU
    leg times the fp32 oracle restatement of the same step (100 reps, median)."""
    from orator_b200 import AsrTextConfig, Layer32
    past_rows, reps = 512, 100
    g = torch.Generator().manual_seed(0)
    past = torch.randn(past_rows, HIDDEN, generator=g).numpy()
    query = torch.randn(1, HIDDEN, generator=g).numpy()
    lay = Layer32(AsrTextConfig(num_layers=1, max_seq_len=past_rows + 16))
    lay.init_synthetic(0, 0)
    lay.forward(past, 0)
    dq = torch.from_numpy(query).cuda()
    dout = torch.empty_like(dq)
    s = torch.cuda.current_stream()
    for _ in range(5):
        lay.truncate(past_rows)
        lay.forward_device(dq.data_ptr(), 1, past_rows, dout.data_ptr(), s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        lay.truncate(past_rows)
        e0.record(s)
        lay.forward_device(dq.data_ptr(), 1, past_rows, dout.data_ptr(), s)
        e1.record(s)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    lay.close()
    us = statistics.median(ts)
    nbytes = 201326592 + (2 * HIDDEN + 256) * 4 + 2 * (past_rows + 1) * 1024 * 4
    out = {"workload": "config1: one fp32 Qwen3-1.7B-shaped layer, decode row at position 512 "
                       "(KV 513 fp32), seed 0, B=1",
           "gpu_us_per_step": us, "bytes_per_step": nbytes,
           "achieved_gbs": nbytes / (us * 1e-6) / 1e9, "frac": nbytes / (us * 1e-6) / 1e9 / hbm,
           "note": "5 launches per row chained by programmatic dependent launch (norm+qkv GEMV, "
                   "attention with q/k norm+RoPE+KV store, o GEMV, norm+gate/up GEMV, down GEMV), median of 100 reps, L2 not flushed"}
    if cpu:
        from oracle import decoder_oracle as D
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        cfg = D.Config(num_layers=1, vocab_size=16, max_seq_len=past_rows + 16)
        o = D.OracleDecoder(cfg, D.synthetic_weights(cfg, 0, bf16=False), quantize=False)
        o.forward(past, 0)
        ct = []
        for _ in range(reps):
            o.truncate(past_rows)
            t0 = time.perf_counter()
            o.forward(query, past_rows)
            ct.append((time.perf_counter() - t0) * 1e6)
        out["cpu_baseline"] = {"us_per_step": statistics.median(ct), "cores": threads,
                               "kind": "port", "sample": "100 decode rows of the fp32 oracle layer"}
    return out


VAD_MACS_PER_WINDOW = (4 * 258 * 256           # STFT (4 frames x 258 filters x 256)
                       + 128 * 4 * 129 * 3       # enc0
                       + 64 * 2 * 128 * 3        # enc1
                       + 64 * 64 * 2             # enc2 (two taps see data)
                       + 128 * 64                # enc3 (centre tap)
                       + 512 * 256 + 128)        # LSTM gates + head


def run_config5(torch, cpu: bool, ref_gpu: bool, reps: int = 3):
    """Config 5: the Silero-shaped detector (seed 4) over 4096 streams x 100
    steps of 512 (+64 context) samples, PCM U[-1, 1) on the device; one step
    of the bench = the whole 409,600-window job (front end of every window,
    then each stream's LSTM scan over its 100 steps). Device time with CUDA
    events; e2e through the C ABI from pinned host PCM to host probabilities."""
    from orator_b200.vad import BatchVad
    S, steps = 4096, 100
    g = torch.Generator(device="cuda").manual_seed(4)
    pcm = torch.rand(S, steps * 512, device="cuda", generator=g) * 2 - 1
    probs = torch.empty(S, steps, device="cuda")
    v = BatchVad(S)
    v.init_synthetic(4)
    s = torch.cuda.current_stream()
    for _ in range(2):
        v.reset()
        v.run_device(pcm.data_ptr(), steps, probs.data_ptr(), s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        v.reset()
        torch.cuda.synchronize()
        e0.record(s)
        v.run_device(pcm.data_ptr(), steps, probs.data_ptr(), s)
        e1.record(s)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ms = statistics.median(ts)
    windows = S * steps
    flops = 2.0 * VAD_MACS_PER_WINDOW * windows
    peak = 148 * 128 * 2 * 1.965e9 / 1e12  # fp32 FMA issue rate, nominal (no measured fp32 peak)
    host = torch.empty(S, steps * 512, pin_memory=True)
    host.copy_(pcm)
    hp = host.numpy()
    v.reset()
    v.run(hp)
    t0 = time.perf_counter()
    v.reset()
    v.run(hp)
    e2e_s = time.perf_counter() - t0
    out = {"workload": "config5: Silero-shaped detector, 4096 streams x 100 steps (512 + 64 samples), "
                       "fp32, seed 4, LSTM state carried across steps",
           "value": windows / (ms * 1e-3), "unit": "windows/s", "ms_per_step": ms,
           "tflops": flops / (ms * 1e-3) / 1e12, "roofline": {
               "bound": "fp32 work (split-bf16 tensor-core MMAs)", "achieved": flops / (ms * 1e-3) / 1e12,
               "peak": peak, "peak_kind": "nominal fp32 issue rate, 148 SM x 128 FMA/clk x 1.965 GHz",
               "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak},
           "e2e": {"value": windows / e2e_s, "unit": "windows/s",
                   "h2d_bytes_per_step": S * steps * 512 * 4, "d2h_bytes_per_step": S * steps * 4}}
    v.close()
    if cpu:
        from oracle import vad_oracle as V
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        Sc, kc = 256, 10
        o = V.BatchVadOracle(V.synthetic_weights(4), Sc)
        x = pcm[:Sc, :kc * 512].cpu().numpy()
        t0 = time.perf_counter()
        o.run(x, kc)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": Sc * kc / dt, "unit": "windows/s", "cores": threads,
                               "kind": "port", "sample": f"{Sc} streams x {kc} steps (numpy restatement)"}
    if ref_gpu:
        out["reference_gpu"] = vad_reference_gpu_rate(pcm)
    return out


TOWER_FRAMES = 1000  # 10 s utterances (100 mel frames per second)


def tower_flops(frames_list, layers: int = 24) -> float:
    """Algorithmic FLOPs of one tower pass over the utterances (2 per MAC):
    the three convolutions at the reference's padded chunk widths, conv_out,
    the encoder layers (q, k, v, out, fc1, fc2 and full attention inside each
    utterance) and proj1 / proj2; kept rows only past conv_out."""
    co = lambda x: 0 if x <= 0 else (x - 1) // 2 + 1
    ol = lambda n: co(co(co(n % 100))) + (n // 100) * 13
    f = 0.0
    for n in frames_list:
        ch = (n + 99) // 100
        mcl = min(n, 100)
        w1, w2, w3 = co(mcl), co(co(mcl)), co(co(co(mcl)))
        f += ch * 2.0 * (64 * w1 * 480 * 9 + 32 * w2 * 480 * 4320 + 16 * w3 * 480 * 4320)
        f += ch * w3 * 2.0 * 7680 * 1024
        r = ol(n)
        f += layers * (2.0 * r * (4 * 1024 * 1024 + 2 * 1024 * 4096) + 4.0 * r * r * 1024)
        f += 2.0 * r * (1024 * 1024 + 1024 * 2048)
    return f


def run_tower(torch, cpu: bool, ref_gpu: bool, utts: int = 64, reps: int = 3):
    """The audio tower (24 layers, seed 5) over `utts` 10 s utterances of
    N(0, 1) log-mel in one batched call (attention per utterance). Device
    time with CUDA events; e2e from pinned host mel to host rows through the
    C ABI's batched call, copies included."""
    from orator_b200.tower import AudioTower, output_length
    frames = [TOWER_FRAMES] * utts
    rows = sum(output_length(n) for n in frames)
    g = torch.Generator(device="cuda").manual_seed(5)
    mel = torch.randn(utts * 128 * TOWER_FRAMES, device="cuda", generator=g)
    out = torch.empty(rows, 2048, device="cuda")
    t = AudioTower(24)
    t.init_synthetic(5)
    s = torch.cuda.current_stream()
    for _ in range(3):
        t.forward_batch(mel.data_ptr(), frames, out.data_ptr(), s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize()
        e0.record(s)
        t.forward_batch(mel.data_ptr(), frames, out.data_ptr(), s)
        e1.record(s)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ms = statistics.median(ts)
    flops = tower_flops(frames)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        peak, kind = 1590.0, "fallback"
    tf = flops / (ms * 1e-3) / 1e12
    audio_s = utts * TOWER_FRAMES / 100.0
    hm = torch.empty(mel.numel(), pin_memory=True)
    hm.copy_(mel)
    ho = torch.empty(rows, 2048, pin_memory=True)
    e2e = []
    for _ in range(reps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        mel.copy_(hm, non_blocking=True)
        t.forward_batch(mel.data_ptr(), frames, out.data_ptr(), s)
        ho.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        e2e.append(time.perf_counter() - t0)
    e2e_s = statistics.median(e2e)
    res = {"workload": f"audio tower: 24 layers (d 1024, 16 heads, ffn 4096) + conv front end, "
                       f"{utts} utterances x {TOWER_FRAMES} mel frames (10 s) in one batched call, "
                       "bf16 GEMMs / fp32 elsewhere, seed 5",
           "value": audio_s / (ms * 1e-3), "unit": "audio seconds/s", "ms_per_step": ms,
           "rows_per_s": rows / (ms * 1e-3),
           "roofline": {"bound": "tensor", "achieved": tf, "peak": peak,
                        "peak_kind": f"{kind} cuBLAS bf16 burst", "unit": "TFLOP/s",
                        "frac": tf / peak, "flops_per_step": flops,
                        "note": "whole pass (all kernels) against the GEMM peak"},
           "e2e": {"value": audio_s / e2e_s, "unit": "audio seconds/s",
                   "h2d_bytes_per_step": mel.numel() * 4, "d2h_bytes_per_step": rows * 2048 * 4}}
    t.close()
    if cpu or ref_gpu:
        from oracle import tower_oracle as TO
        from orator_b200 import synth_f32

        def gpu_normal(seed, tid, n, std, mean):
            buf = torch.empty(n, dtype=torch.float32, device="cuda")
            synth_f32(buf.data_ptr(), n, seed, tid, std, mean, False)
            return buf.cpu().numpy()
        w = TO.synthetic_weights(24, normal=gpu_normal)
        sample = mel[:128 * TOWER_FRAMES].view(128, TOWER_FRAMES).cpu().numpy()
        if cpu:
            threads = os.cpu_count() or 1
            torch.set_num_threads(threads)
            o = TO.TowerOracle(w, 24)
            k = 2
            t0 = time.perf_counter()
            for _ in range(k):
                o.forward(sample)
            dt = time.perf_counter() - t0
            res["cpu_baseline"] = {"value": k * TOWER_FRAMES / 100.0 / dt, "unit": "audio seconds/s",
                                   "cores": threads, "kind": "port",
                                   "sample": f"{k} x one 10 s utterance (torch fp32 restatement)"}
        if ref_gpu:
            res["reference_gpu"] = tower_reference_gpu_rate(w, sample)
            if "value" in res["reference_gpu"]:
                res["reference_gpu"]["ours_over_reference"] = res["value"] / res["reference_gpu"]["value"]
    return res


def tower_reference_gpu_rate(weights, mel, utts: int = 8):
    """The reference's own AsrAudioTower (oracle/_ref) on this GPU through its
    public host-to-host Forward, one 10 s utterance per call as it is built."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libref_asr.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref/libref_asr.so not built (oracle/build_ref.sh)"}
    import ctypes as C
    import shutil
    from oracle import tower_oracle as TO
    d = tempfile.mkdtemp(prefix="ref_tower_")
    try:
        TO.write_checkpoint(d, weights, 24)
        L = C.CDLL(lib_path)
        L.ref_tower_create.restype = C.c_void_p
        L.ref_tower_create.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_tower_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.ref_tower_destroy.argtypes = [C.c_void_p]
        h = C.c_void_p(L.ref_tower_create(d.encode(), 24, 0))
        if not h:
            return {"unavailable": "reference tower failed to load"}
        n = mel.shape[1]
        x = np.ascontiguousarray(mel, np.float32)
        out = np.empty((TO.output_length(n), 2048), np.float32)
        for _ in range(2):
            L.ref_tower_forward(h, x.ctypes.data_as(C.c_void_p), C.c_int(n), out.ctypes.data_as(C.c_void_p))
        t0 = time.perf_counter()
        for _ in range(utts):
            L.ref_tower_forward(h, x.ctypes.data_as(C.c_void_p), C.c_int(n), out.ctypes.data_as(C.c_void_p))
        dt = time.perf_counter() - t0
        L.ref_tower_destroy(h)
        return {"value": utts * n / 100.0 / dt, "unit": "audio seconds/s",
                "sample": f"{utts} calls of AsrAudioTower::Forward on one 10 s utterance "
                          "(host mel in, host rows out)"}
    finally:
        shutil.rmtree(d, ignore_errors=True)


SF_CHUNK_FRAMES, SF_CACHE = 341 * 8, 376  # 340-frame chunk + 1 right context; spkcache + FIFO


def sortformer_flops(n_frames: int = SF_CHUNK_FRAMES, n_cache: int = SF_CACHE,
                     conf_layers: int = 17, dec_layers: int = 18) -> float:
    """Algorithmic fp32 FLOPs (2 per MAC) of one streaming step: the
    pre-encode convolutions and Linear, the conformer stack (attention counted
    over the T x T scores it uses) and the decoder with its head."""
    cl = lambda x: (x + 2 - 3) // 2 + 1
    h0 = cl(n_frames)
    h1 = cl(h0)
    h2 = cl(h1)
    T = n_cache + h2
    P = 2 * T - 1
    macs = h0 * 64 * 256 * 9 + h1 * 32 * 256 * (9 + 256) + h2 * 16 * 256 * (9 + 256) + h2 * 4096 * 512
    lay = (2 * T * 512 * 2048 * 2 + T * 512 * 1536 + P * 512 * 512 + 8 * T * T * 64 * 3
           + T * 512 * 512 + T * 512 * 1024 + T * 512 * 9 + T * 512 * 512)
    dec = T * 192 * 576 + 8 * T * T * 24 * 2 + T * 192 * 192 + 2 * T * 192 * 768
    macs += conf_layers * lay + T * 512 * 192 + dec_layers * dec + T * 192 * 192 + T * 192 * 4
    return 2.0 * macs


def run_config4(torch, cpu: bool, ref_gpu: bool, reps: int = 5):
    """Config 4: one streaming Sortformer step (17 FastConformer + 18
    transformer layers, fp32, seed 3): pre-encode of a 2728-frame N(0, 1)
    log-mel chunk (340 + 1 frames after 8x subsampling) behind 376 speaker-cache
    + FIFO rows, T = 717, the encoder, decoder and speaker head. Device time with
    CUDA events; e2e through the C ABI from host mel and cache to host
    probabilities."""
    from orator_b200.sortformer import Sortformer
    g = torch.Generator(device="cuda").manual_seed(3)
    mel = torch.randn(128 * SF_CHUNK_FRAMES, device="cuda", generator=g)
    cache = torch.randn(SF_CACHE * 512, device="cuda", generator=g)
    T = SF_CACHE + 341
    preds = torch.empty(T, 4, device="cuda")
    m = Sortformer(17, 18)
    m.init_synthetic(3)
    s = torch.cuda.current_stream()
    for _ in range(3):
        m.step_device(mel.data_ptr(), SF_CHUNK_FRAMES, SF_CHUNK_FRAMES, cache.data_ptr(), SF_CACHE,
                      preds.data_ptr(), s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize()
        e0.record(s)
        m.step_device(mel.data_ptr(), SF_CHUNK_FRAMES, SF_CHUNK_FRAMES, cache.data_ptr(), SF_CACHE,
                      preds.data_ptr(), s)
        e1.record(s)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ms = statistics.median(ts)
    flops = sortformer_flops()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16, kind = float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        bf16, kind = 1590.0, "fallback"
    peak = bf16 / 3.0
    tf = flops / (ms * 1e-3) / 1e12
    hm, hc = mel.cpu().numpy().reshape(128, SF_CHUNK_FRAMES), cache.cpu().numpy().reshape(SF_CACHE, 512)
    m.step(hm, hc)
    e2e = []
    for _ in range(reps):
        t0 = time.perf_counter()
        m.step(hm, hc)
        e2e.append(time.perf_counter() - t0)
    e2e_s = statistics.median(e2e)
    audio = 340 * 0.08  # seconds of audio one step advances (chunk_len x 80 ms frames)
    res = {"workload": "config4: streaming Sortformer step, 17 FastConformer (d 512) + 18 transformer "
                       "(d 192) layers, fp32 weights (seed 3), 2728-frame chunk + 376 cache/FIFO rows, T=717",
           "value": 1e3 / ms, "unit": "steps/s", "ms_per_step": ms,
           "audio_seconds_per_s": audio * 1e3 / ms,
           "roofline": {"bound": "tensor (fp32 as 3 bf16 products)", "achieved": tf, "peak": peak,
                        "peak_kind": f"{kind} cuBLAS bf16 burst / 3", "unit": "TFLOP/s",
                        "frac": tf / peak, "flops_per_step": flops,
                        "nominal_fp32_simt_tflops": 148 * 128 * 2 * 1.965e9 / 1e12},
           "e2e": {"value": 1.0 / e2e_s, "unit": "steps/s",
                   "h2d_bytes_per_step": (128 * SF_CHUNK_FRAMES + SF_CACHE * 512) * 4,
                   "d2h_bytes_per_step": T * 4 * 4}}
    m.close()
    if cpu or ref_gpu:
        from oracle import sortformer_oracle as SO
        from orator_b200 import synth_f32

        def gpu_normal(seed, tid, n, std, mean):
            buf = torch.empty(n, dtype=torch.float32, device="cuda")
            synth_f32(buf.data_ptr(), n, seed, tid, std, mean, False)
            return buf.cpu().numpy()
        w = SO.synthetic_weights(17, 18, normal=gpu_normal)
        if cpu:
            threads = os.cpu_count() or 1
            torch.set_num_threads(threads)
            o = SO.SortformerOracle(w, 17, 18)
            t0 = time.perf_counter()
            emb, t2, v2 = o.pre_encode(hm, SF_CHUNK_FRAMES)
            o.encode_decode(np.concatenate([hc, emb]), SF_CACHE + v2)
            dt = time.perf_counter() - t0
            res["cpu_baseline"] = {"value": 1.0 / dt, "unit": "steps/s", "cores": threads, "kind": "port",
                                   "sample": "one full step (torch fp32 restatement)"}
        if ref_gpu:
            res["reference_gpu"] = sortformer_reference_gpu_rate(w, hm, hc)
            if "value" in res["reference_gpu"]:
                res["reference_gpu"]["ours_over_reference"] = res["value"] / res["reference_gpu"]["value"]
    return res


def sortformer_reference_gpu_rate(weights, mel, cache, steps: int = 3):
    """The reference's own ConformerPreEncode / ConformerLayer x 17 /
    SortformerDecoder (oracle/_ref) on this GPU, one step per call through
    their public host-to-host Forward methods."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libref_asr.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref/libref_asr.so not built (oracle/build_ref.sh)"}
    import ctypes as C
    import shutil
    from oracle import sortformer_oracle as SO
    d = tempfile.mkdtemp(prefix="ref_sf_")
    try:
        path = SO.write_safetensors(os.path.join(d, "sf.safetensors"), weights, 17, 18)
        L = C.CDLL(lib_path)
        L.ref_sf_create.restype = C.c_void_p
        L.ref_sf_create.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_sf_destroy.argtypes = [C.c_void_p]
        L.ref_sf_preencode.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                       C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ref_sf_encdec.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        h = C.c_void_p(L.ref_sf_create(path.encode(), 17, 18))
        if not h:
            return {"unavailable": "reference Sortformer failed to load"}
        n = mel.shape[1]
        x = np.ascontiguousarray(mel, np.float32)
        emb = np.empty((341, 512), np.float32)
        preds = np.empty((SF_CACHE + 341, 4), np.float32)
        t2, v2 = C.c_int(), C.c_int()

        def one():
            L.ref_sf_preencode(h, x.ctypes.data_as(C.c_void_p), 128, n, n,
                               emb.ctypes.data_as(C.c_void_p), C.byref(t2), C.byref(v2))
            cat = np.ascontiguousarray(np.concatenate([cache, emb]), np.float32)
            L.ref_sf_encdec(h, cat.ctypes.data_as(C.c_void_p), cat.shape[0], SF_CACHE + v2.value,
                            preds.ctypes.data_as(C.c_void_p))
        one()
        t0 = time.perf_counter()
        for _ in range(steps):
            one()
        dt = time.perf_counter() - t0
        L.ref_sf_destroy(h)
        return {"value": steps / dt, "unit": "steps/s",
                "sample": f"{steps} steps of ConformerPreEncode::Forward + ForwardEncoderDecoder "
                          "(host in, host out)"}
    finally:
        shutil.rmtree(d, ignore_errors=True)


def vad_reference_gpu_rate(pcm, streams: int = 16):
    """The reference's own GpuVad (oracle/_ref) on this GPU: one stream at a
    time, as it is built, for a sample of streams x all 100 steps (its
    DebugWindowProbs: one batched pass over the stream's windows)."""
    import ctypes as C
    import shutil
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libref_asr.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref/libref_asr.so not built (oracle/build_ref.sh)"}
    from oracle import vad_oracle as V
    L = C.CDLL(lib_path)
    L.ref_gpuvad_create.restype = C.c_void_p
    L.ref_gpuvad_create.argtypes = [C.c_char_p]
    d = tempfile.mkdtemp(prefix="ref_vad_")
    try:
        path = V.write_safetensors(os.path.join(d, "vad.safetensors"), V.synthetic_weights(4))
        h = C.c_void_p(L.ref_gpuvad_create(path.encode()))
        x = pcm[:streams].cpu().numpy()
        steps = x.shape[1] // 512
        out = np.zeros(steps, np.float32)
        L.ref_gpuvad_probs(h, x[0].ctypes.data_as(C.c_void_p), C.c_int(x.shape[1]),
                           out.ctypes.data_as(C.c_void_p))  # warm-up
        t0 = time.perf_counter()
        for s in range(streams):
            L.ref_gpuvad_probs(h, x[s].ctypes.data_as(C.c_void_p), C.c_int(x.shape[1]),
                               out.ctypes.data_as(C.c_void_p))
        dt = time.perf_counter() - t0
        L.ref_gpuvad_destroy(h)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"value": streams * steps / dt, "unit": "windows/s",
            "sample": f"{streams} streams x {steps} steps, one stream per call (wall clock, "
                      "each call synchronizes)"}


def measure_prefill(dec, torch, prompt, s, reps=5):
    """Config 2's 400-row prefill from device-resident rows (tcgen05 GEMMs,
    flash prefill attention, last-row lm_head), device time per prefill, and
    its arithmetic rate against the measured bf16 GEMM peak."""
    d_prompt = torch.from_numpy(prompt).cuda()
    for _ in range(2):
        dec.ResetCache()
        dec.PrefillAtDevice(d_prompt.data_ptr(), PROMPT_ROWS, 0, s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        dec.ResetCache()
        dec.PrefillAtDevice(d_prompt.data_ptr(), PROMPT_ROWS, 0, s)
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    layer_params = (4096 + 2048 + 12288) * 2048 + 2048 * 6144  # qkv, o, gate/up, down
    flops = (2 * PROMPT_ROWS * LAYERS * layer_params          # projections
             + 4 * LAYERS * 16 * 128 * PROMPT_ROWS * (PROMPT_ROWS + 1) // 2  # causal attention
             + 2 * VOCAB * HIDDEN)                              # last-row lm_head
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        peak = 1590.0
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": "config2 prefill: 400 rows (375 audio + 25 token embeddings), 28 layers",
            "ms": ms, "tflops": tf, "flops": flops, "bf16_peak_tflops": peak, "frac": tf / peak,
            "note": "device-resident rows, CUDA events, mean of 5"}


def run_ours(args):
    import torch
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        # a rank that fails ends the others' next collective within 2 minutes
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    from orator_b200 import AsrTextConfig, AsrTextDecoder

    dec = AsrTextDecoder(AsrTextConfig(max_seq_len=2816))  # room for config 3's longest session
    dec.init_synthetic(SEED)
    prompt = build_prompt_gpu(dec, torch)
    dec.ResetCache()
    dec.Prefill(prompt)

    def step():
        dec.TruncateCache(PROMPT_ROWS)
        # ban_steps 0 and no EOS ids: every step decodes exactly 128 tokens
        return dec.DecodeGreedy(PROMPT_ROWS, NEW_TOKENS, -1, -1, ban_steps=0, batch=NEW_TOKENS)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    with sampler:
        e0.record(s)
        for _ in range(args.steps):
            toks = step()
        e1.record(s)
        barrier()
    ms = e0.elapsed_time(e1)
    clocks = sampler.summary()

    # end to end through the public API: host prompt in (H2D), host tokens out (D2H)
    for _ in range(1):
        dec.ResetCache(); dec.Prefill(prompt); dec.DecodeGreedy(PROMPT_ROWS, NEW_TOKENS, -1, -1, 0, 32)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s)
    for _ in range(args.steps):
        dec.ResetCache()
        dec.Prefill(prompt)
        dec.DecodeGreedy(PROMPT_ROWS, NEW_TOKENS, -1, -1, ban_steps=0, batch=32)
    f1.record(s)
    barrier()
    e2e_ms = f0.elapsed_time(f1)

    prof = dec.profile_kernels(iters=20)
    ref_gpu = (reference_gpu_rate(prompt) if world == 1 and not args.no_reference_gpu
               else None)
    prefill = measure_prefill(dec, torch, prompt, s)
    ragged = None if args.no_ragged else run_ragged(dec, torch, world, dist, rank, steps=args.ragged_steps)
    ragged_strong = (run_ragged(dec, torch, world, dist, rank, strong=True, steps=args.ragged_steps)
                     if world > 1 and not args.no_ragged else None)
    if dist:
        t = torch.tensor([ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    tokens = NEW_TOKENS * args.steps * world
    value = tokens / (ms / 1e3)
    hbm, peak_kind = peaks()
    lm_bytes = VOCAB * HIDDEN * 2 + HIDDEN * 4
    lm_gbs = lm_bytes / (prof["lm_head"] * 1e-3) / 1e9
    mean_s = PROMPT_ROWS + (NEW_TOKENS + 1) / 2
    step_bytes = WEIGHT_BYTES + KV_BYTES_PER_POS * mean_s
    tok_ms = ms / (NEW_TOKENS * args.steps)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, seeded N(0,1) audio rows)",
        "config": {"workload": WORKLOAD2,
                   "global_batch": world, "parallelism": f"replicas x{world} (independent sessions)",
                   "l2": "inputs larger than L2 (3.44 GB of weights streamed per token)"},
        "per_token_ms": tok_ms,
        "step_hbm": {"bytes_per_token": step_bytes, "achieved_gbs": step_bytes / (tok_ms * 1e-3) / 1e9,
                     "frac": step_bytes / (tok_ms * 1e-3) / 1e9 / hbm},
        "roofline": {"bound": "hbm",
                     "kernel": "decode_mk_kernel (one cooperative launch = 128 tokens x 28 layers + lm_head)",
                     "achieved": step_bytes * NEW_TOKENS / (ms / args.steps * 1e-3) / 1e9,
                     "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": step_bytes * NEW_TOKENS / (ms / args.steps * 1e-3) / 1e9 / hbm,
                     # ncu dram__bytes_read+write of a 4-token launch (config 2,
                     # KV 401..404) = 3.4924 GB per token, scaled to this launch
                     "traffic": NCU_BYTES_PER_TOKEN * NEW_TOKENS,
                     "algorithmic_bytes_per_launch": step_bytes * NEW_TOKENS,
                     "gemv_kernel_lm_head": {"achieved_gbs": lm_gbs, "frac": lm_gbs / hbm,
                                             "note": "per-kernel path, 622 MB launch, CUDA events"},
                     "per_class_ms_per_kernel_path": prof},
        "e2e": {"value": NEW_TOKENS * args.steps * world / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": PROMPT_ROWS * HIDDEN * 4,
                "d2h_bytes_per_step": NEW_TOKENS * 4,
                "note": "per step: Prefill(host 400x2048 fp32) + DecodeGreedy(128, batch 32) through the C ABI"},
        "gpu_launches": args.steps * 2,  # seed argmax + one persistent decode launch per step
        "prefill": prefill,
        "clocks": clocks,
    }
    if ref_gpu is not None:
        if "value" in ref_gpu:
            ref_gpu["ours_over_reference"] = value / ref_gpu["value"]
        line["reference_gpu"] = ref_gpu
    if ragged is not None:
        line["ragged"] = ragged
    if ragged_strong is not None:
        line["ragged_strong"] = ragged_strong
    if not args.no_config1:
        line["config1"] = run_config1(torch, hbm, cpu=world == 1 and not args.no_cpu_baseline)
    if world == 1 and not args.no_config5:
        line["config5"] = run_config5(torch, cpu=not args.no_cpu_baseline,
                                      ref_gpu=not args.no_reference_gpu)
    if world == 1 and not args.no_config4:
        line["config4"] = run_config4(torch, cpu=not args.no_cpu_baseline,
                                      ref_gpu=not args.no_reference_gpu)
    if world == 1 and not args.no_tower:
        line["tower"] = run_tower(torch, cpu=not args.no_cpu_baseline,
                                  ref_gpu=not args.no_reference_gpu)
    if world == 1 and not args.no_cpu_baseline:
        rate, threads, _ = cpu_oracle_rate(args.cpu_sample)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{args.cpu_sample} greedy decode tokens at KV 401.. "
                                          "after a 400-row prefill (oracle restatement, fp32 torch)"}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ragged", action="store_true", help="skip the config-3 ragged batch run")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own CUDA decoder (oracle/_ref)")
    ap.add_argument("--no-config1", action="store_true", help="skip the config-1 fp32 layer run")
    ap.add_argument("--no-config5", action="store_true", help="skip the config-5 detector run")
    ap.add_argument("--config1-only", action="store_true",
                    help="run only the config-1 fp32 layer timing (profiling)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only config 2's 400-row prefill timing (profiling)")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 Sortformer run")
    ap.add_argument("--config4-only", action="store_true",
                    help="run only the config-4 Sortformer step (profiling)")
    ap.add_argument("--no-tower", action="store_true", help="skip the audio tower run")
    ap.add_argument("--tower-only", type=int, default=0, metavar="UTTS",
                    help="run only the audio tower leg over UTTS utterances (profiling)")
    ap.add_argument("--ragged-steps", type=int, default=256,
                    help="decode steps of the config-3 runs (256 = the config; fewer for profiling)")
    ap.add_argument("--tokens", type=int, default=128,
                    help="decode tokens per step (128 = config 2; smaller only for profiler runs)")
    args = ap.parse_args()
    global NEW_TOKENS
    NEW_TOKENS = args.tokens
    if args.impl == "reference":
        run_reference(args)
        return
    if args.config4_only:
        import torch
        print(json.dumps(run_config4(torch, cpu=False, ref_gpu=False)), flush=True)
        return
    if args.config1_only:
        import torch
        print(json.dumps(run_config1(torch, peaks()[0], cpu=False)), flush=True)
        return
    if args.prefill_only:
        import torch
        from orator_b200 import AsrTextConfig, AsrTextDecoder
        dec = AsrTextDecoder(AsrTextConfig(max_seq_len=2816))
        dec.init_synthetic(SEED)
        prompt = build_prompt_gpu(dec, torch)
        print(json.dumps(measure_prefill(dec, torch, prompt, torch.cuda.current_stream())), flush=True)
        return
    if args.tower_only:
        import torch
        print(json.dumps(run_tower(torch, cpu=False, ref_gpu=False, utts=args.tower_only)), flush=True)
        return
    try:
        run_ours(args)
    except BaseException:
        import traceback
        rank = dist_env()[0]
        sys.stderr.write(f"[rank {rank}] bench failed:\n{traceback.format_exc()}")
        sys.stderr.flush()
        raise


if __name__ == "__main__":
    main()
