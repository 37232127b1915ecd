"""ctypes access to the reference decoder built by oracle/build_ref.sh
(oracle/_ref/libref_asr.so). Test infrastructure: a checker, never the product."""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_asr.so")


def available() -> bool:
    return os.path.exists(LIB)


class RefDecoder:
    def __init__(self, model_dir: str, num_layers: int, vocab: int, max_seq: int = 2048,
                 graphs: bool = False):
        L = C.CDLL(LIB)
        for f in ("ref_create", "ref_create_graphs"):
            getattr(L, f).restype = C.c_void_p
            getattr(L, f).argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int]
        L.ref_last_error.restype = C.c_char_p
        for f in ["ref_prefill_at", "ref_copy_logits", "ref_decode_step_token", "ref_argmax",
                  "ref_destroy", "ref_truncate", "ref_cache_len", "ref_decode_greedy"]:
            getattr(L, f).argtypes = None
        self.L, self.vocab = L, vocab
        h = (L.ref_create_graphs if graphs else L.ref_create)(model_dir.encode(), num_layers,
                                                               vocab, max_seq)
        if not h:
            raise RuntimeError(L.ref_last_error().decode())
        self.h = C.c_void_p(h)

    def prefill_at(self, x, pos0):
        x = np.ascontiguousarray(x, np.float32)
        assert self.L.ref_prefill_at(self.h, x.ctypes.data_as(C.c_void_p), C.c_int(x.shape[0]),
                                     C.c_int(pos0)) == 0
        return self.logits()

    def logits(self):
        out = np.empty(self.vocab, np.float32)
        assert self.L.ref_copy_logits(self.h, out.ctypes.data_as(C.c_void_p)) == 0
        return out

    def decode_step(self, tok, pos):
        assert self.L.ref_decode_step_token(self.h, C.c_int(tok), C.c_int(pos)) == 0
        return self.logits()

    def close(self):
        if self.h:
            self.L.ref_destroy(self.h)
            self.h = None


class RefOps:
    """The reference's own free operators (asr_ops / asr_gemm), unmodified,
    on device pointers (ints); each call synchronizes the device."""

    def __init__(self):
        self.L = C.CDLL(LIB)
        self.L.ref_last_error.restype = C.c_char_p

    def _ok(self, rc):
        if rc != 0:
            raise RuntimeError(self.L.ref_last_error().decode())

    def rms_norm(self, x, w, out, rows, dim, eps):
        self._ok(self.L.ref_op_rmsnorm(C.c_void_p(x), C.c_void_p(w), C.c_void_p(out), rows, dim,
                                       C.c_float(eps)))

    def rope_half(self, x, pos, n, heads, dim, theta):
        self._ok(self.L.ref_op_rope_half(C.c_void_p(x), C.c_void_p(pos), n, heads, dim,
                                         C.c_float(theta)))

    def rope_interleaved(self, x, pos, n, heads, dim, theta):
        self._ok(self.L.ref_op_rope_interleaved(C.c_void_p(x), C.c_void_p(pos), n, heads, dim,
                                                C.c_float(theta)))

    def swiglu(self, g, u, out, n):
        self._ok(self.L.ref_op_swiglu(C.c_void_p(g), C.c_void_p(u), C.c_void_p(out), n))

    def gqa(self, q, k, v, out, T, hq, hkv, dh, scale, causal):
        self._ok(self.L.ref_op_gqa(C.c_void_p(q), C.c_void_p(k), C.c_void_p(v), C.c_void_p(out),
                                   T, hq, hkv, dh, C.c_float(scale), int(causal)))

    def argmax_banned(self, x, n, ban0, ban1, out):
        self._ok(self.L.ref_op_argmax_banned(C.c_void_p(x), n, ban0, ban1, C.c_void_p(out)))

    def f32_to_bf16(self, x, out, n):
        self._ok(self.L.ref_op_f32_to_bf16(C.c_void_p(x), C.c_void_p(out), C.c_long(n)))

    def linear(self, x, w, bias, out, M, K, N, act):
        self._ok(self.L.ref_op_linear(C.c_void_p(x), C.c_void_p(w), C.c_void_p(bias or 0),
                                      C.c_void_p(out), M, K, N, act))


class RefTower:
    """The reference's AsrAudioTower (src/model/asr_audio_tower.cu), unmodified,
    loaded from a safetensors directory; forward is its host-to-host Forward."""

    def __init__(self, model_dir: str, layers: int, windowed: bool = False):
        L = C.CDLL(LIB)
        L.ref_tower_create.restype = C.c_void_p
        L.ref_tower_create.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_tower_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.ref_tower_destroy.argtypes = [C.c_void_p]
        L.ref_last_error.restype = C.c_char_p
        h = L.ref_tower_create(model_dir.encode(), layers, 1 if windowed else 0)
        if not h:
            raise RuntimeError(L.ref_last_error().decode())
        self.L, self.h = L, C.c_void_p(h)

    def forward(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        n = mel.shape[1]
        rows = self.L.ref_tower_output_length(C.c_int(n))
        out = np.empty((max(rows, 1), 2048), np.float32)
        got = self.L.ref_tower_forward(self.h, mel.ctypes.data_as(C.c_void_p), C.c_int(n),
                                       out.ctypes.data_as(C.c_void_p))
        if got < 0:
            raise RuntimeError(self.L.ref_last_error().decode())
        return out[:got]

    def close(self):
        if self.h:
            self.L.ref_tower_destroy(self.h)
            self.h = None


class RefSortformer:
    """The reference's ConformerPreEncode / ConformerLayer / SortformerDecoder
    (src/model/conformer_preencode.cu, conformer_layer.cu, sortformer_decoder.cu),
    unmodified, from one F32 safetensors file."""

    def __init__(self, path: str, conf_layers: int, dec_layers: int):
        L = C.CDLL(LIB)
        L.ref_sf_create.restype = C.c_void_p
        L.ref_sf_create.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_sf_destroy.argtypes = [C.c_void_p]
        L.ref_sf_preencode.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ref_sf_encdec.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.ref_last_error.restype = C.c_char_p
        h = L.ref_sf_create(path.encode(), conf_layers, dec_layers)
        if not h:
            raise RuntimeError(L.ref_last_error().decode())
        self.L, self.h = L, C.c_void_p(h)

    def pre_encode(self, mel, valid):
        mel = np.ascontiguousarray(mel, np.float32)
        n = mel.shape[1]
        T2 = n
        for _ in range(3):
            T2 = (T2 + 2 - 3) // 2 + 1
        out = np.empty((T2, 512), np.float32)
        t, v = C.c_int(), C.c_int()
        assert self.L.ref_sf_preencode(self.h, mel.ctypes.data_as(C.c_void_p), 128, n, valid,
                                       out.ctypes.data_as(C.c_void_p), C.byref(t), C.byref(v)) == 0
        assert t.value == T2
        return out, v.value

    def encode_decode(self, emb, valid):
        emb = np.ascontiguousarray(emb, np.float32)
        T = emb.shape[0]
        out = np.empty((T, 4), np.float32)
        assert self.L.ref_sf_encdec(self.h, emb.ctypes.data_as(C.c_void_p), T, valid,
                                    out.ctypes.data_as(C.c_void_p)) == 0
        return out

    def close(self):
        if self.h:
            self.L.ref_sf_destroy(self.h)
            self.h = None
