"""Seeded synthetic checkpoint files (oracle/st_writer.py's layout) whose
tensors come from orx_synth_f32 on the GPU, which is bit-exact with
oracle/synth.py (tests/test_gpu_decoder.py::test_synth_bit_exact): a
28-layer checkpoint takes seconds instead of the minutes numpy needs.
Test infrastructure only: it feeds the reference build in oracle/_ref."""
import numpy as np

from oracle import st_writer, synth


def gpu_bits(seed, tid, shape, is_norm):
    import torch
    from orator_b200 import synth_f32
    n = int(np.prod(shape))
    buf = torch.empty(n, dtype=torch.float32, device="cuda")
    synth_f32(buf.data_ptr(), n, seed, tid, synth.NORM_STD if is_norm else synth.MATRIX_STD,
              1.0 if is_norm else 0.0, True)
    # bf16-rounded values: the top 16 bits are the bf16 pattern
    return (buf.view(torch.int32) >> 16).to(torch.int16).cpu().numpy().view(np.uint16).reshape(shape)


def write_model(out_dir: str, seed: int, layers: int, vocab: int) -> str:
    return st_writer.write_synthetic_model(out_dir, seed, layers, vocab, shards=4, gen=gpu_bits)
