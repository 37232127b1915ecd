"""Write synthetic weights as a sharded safetensors directory in the layout the
reference loader reads (``model.safetensors.index.json`` with a ``weight_map``
naming each tensor's shard; ``src/io/sharded_safetensor.cc:22-60``).

TEST INFRASTRUCTURE: used only to feed the reference decoder build in
``oracle/_ref`` with the same weights this repository's decoder loads.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from . import synth


def write_shard(path: str, tensors: list[tuple[str, np.ndarray]]):
    """tensors: (name, uint16 bf16 bit array)."""
    header, off = {}, 0
    for name, arr in tensors:
        n = arr.nbytes
        header[name] = {"dtype": "BF16", "shape": list(arr.shape),
                        "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header).encode()
    hj += b" " * ((-len(hj)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for _, arr in tensors:
            f.write(np.ascontiguousarray(arr).tobytes())


def write_synthetic_model(out_dir: str, seed: int, num_layers: int, vocab: int,
                          shards: int = 2, gen=None) -> str:
    """``gen(seed, tid, shape, is_norm)`` may supply each tensor's bf16 bit
    array (e.g. from the bit-exact GPU generator); by default numpy makes it."""
    os.makedirs(out_dir, exist_ok=True)
    items = list(synth.model_tensors(seed, num_layers, vocab))
    groups = [items[i::shards] for i in range(shards)]
    wmap = {}
    for s, g in enumerate(groups):
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        tens = []
        for name, tid, shape, is_norm in g:
            if gen is not None:
                bits = gen(seed, tid, shape, is_norm)
            else:
                v = synth.make_tensor(seed, tid, shape, is_norm, bf16=False)
                bits = synth.f32_to_bf16_bits(v).reshape(shape)
            tens.append((name, bits))
            wmap[name] = fname
        write_shard(os.path.join(out_dir, fname), tens)
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wmap}, f)
    return out_dir
