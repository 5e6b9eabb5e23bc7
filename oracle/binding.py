"""ctypes binding of ``liboracle.so`` (test infrastructure only).

Functions take and return numpy arrays; each wraps one oracle function, which
itself restates one reference function (see ``oracle.h`` for the file:line).
"""
import ctypes as C
import os
import subprocess

import numpy as np

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(ORACLE_DIR, "liboracle.so")

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i32p = C.POINTER(C.c_int32)


class Dims(C.Structure):
    """``orc_dims``: the reference's Transformer plus its hard-coded sizes."""

    _fields_ = [
        ("n_layers", C.c_int32), ("embed_dim", C.c_int32), ("head_dim", C.c_int32),
        ("q_heads", C.c_int32), ("kv_heads", C.c_int32), ("ffn_dim", C.c_int32),
        ("vocab", C.c_int32), ("base_freq", C.c_float), ("mode", C.c_int32),
    ]


def build_oracle():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


def _ptr(a, t):
    return a.ctypes.data_as(t)


class Oracle:
    def __init__(self, path=_LIB_PATH):
        if not os.path.exists(path):
            build_oracle()
        lib = C.CDLL(path)
        self.lib = lib
        sig = {
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "orc_dot_prod_f32": (C.c_float, [_f32p, _f32p, C.c_size_t]),
            "orc_dot_prod_q8": (C.c_float, [_f32p, _u8p, C.c_size_t]),
            "orc_dot_prod_act_q8": (C.c_float, [_u8p, _u8p, C.c_size_t]),
            "orc_q8_matmul": (None, [_f32p, _u8p, _f32p, C.c_size_t, C.c_size_t]),
            "orc_q8_act_matmul": (None, [_u8p, _u8p, _f32p, C.c_size_t, C.c_size_t]),
            "orc_activated_q8": (None, [_f32p, C.c_size_t, _u8p]),
            "orc_q8_dequant": (None, [_u8p, C.c_size_t, _f32p]),
            "orc_rmsnorm": (None, [_f32p, _f32p, _f32p, C.c_size_t]),
            "orc_softmax": (None, [_f32p, _f32p, C.c_size_t]),
            "orc_swiglu": (None, [_f32p, _u8p, _u8p, _u8p, _f32p, C.c_size_t, C.c_size_t]),
            "orc_rope_angles": (None, [C.c_float, C.c_size_t, C.c_size_t, _f32p]),
            "orc_rope": (None, [_f32p, C.c_size_t, _f32p, C.c_size_t, _f32p, C.c_size_t]),
            "orc_embed": (None, [C.c_size_t, _u8p, C.c_size_t, _f32p]),
            "orc_sample": (C.c_size_t, [_f32p, C.c_size_t]),
            "orc_cache_new": (C.c_void_p, []),
            "orc_cache_free": (None, [C.c_void_p]),
            "orc_cache_len": (C.c_size_t, [C.c_void_p]),
            "orc_forward": (C.c_int, [C.POINTER(Dims), C.POINTER(C.c_void_p), C.c_void_p,
                                      _f32p, C.c_size_t, _f32p, _f32p, _f32p]),
            "orc_generate_capped": (C.c_int, [C.POINTER(Dims), C.POINTER(C.c_void_p), _i32p,
                                              C.c_size_t, C.c_size_t, _i32p, _f32p]),
            "orc_set_threads": (None, [C.c_int]),
            "orc_set_fast": (None, [C.c_int]),
            "orc_set_attn_dump": (None, [C.c_void_p]),
            "orc_get_threads": (C.c_int, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args

    # ---- scalar / op level -------------------------------------------------
    def f16_to_f32(self, h):
        return self.lib.orc_f16_to_f32(int(h))

    def f32_to_f16(self, f):
        return self.lib.orc_f32_to_f16(float(f))

    def dot_prod_f32(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        return self.lib.orc_dot_prod_f32(_ptr(a, _f32p), _ptr(b, _f32p), a.size)

    def dot_prod_q8(self, a, blocks):
        a = np.ascontiguousarray(a, np.float32)
        blocks = np.ascontiguousarray(blocks, np.uint8)
        return self.lib.orc_dot_prod_q8(_ptr(a, _f32p), _ptr(blocks, _u8p), a.size)

    def dot_prod_act_q8(self, a_blocks, b_blocks):
        a = np.ascontiguousarray(a_blocks, np.uint8)
        b = np.ascontiguousarray(b_blocks, np.uint8)
        return self.lib.orc_dot_prod_act_q8(_ptr(a, _u8p), _ptr(b, _u8p), a.size // 34 * 32)

    def q8_matmul(self, a, blocks, n):
        a = np.ascontiguousarray(a, np.float32)
        blocks = np.ascontiguousarray(blocks, np.uint8)
        out = np.empty(n, np.float32)
        self.lib.orc_q8_matmul(_ptr(a, _f32p), _ptr(blocks, _u8p), _ptr(out, _f32p), n, a.size)
        return out

    def q8_act_matmul(self, a_blocks, blocks, n):
        a = np.ascontiguousarray(a_blocks, np.uint8)
        blocks = np.ascontiguousarray(blocks, np.uint8)
        out = np.empty(n, np.float32)
        k = a.size // 34 * 32
        self.lib.orc_q8_act_matmul(_ptr(a, _u8p), _ptr(blocks, _u8p), _ptr(out, _f32p), n, k)
        return out

    def activated_q8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 32 * 34, np.uint8)
        self.lib.orc_activated_q8(_ptr(x, _f32p), x.size, _ptr(out, _u8p))
        return out

    def q8_dequant(self, blocks):
        blocks = np.ascontiguousarray(blocks, np.uint8)
        nb = blocks.size // 34
        out = np.empty(nb * 32, np.float32)
        self.lib.orc_q8_dequant(_ptr(blocks, _u8p), nb, _ptr(out, _f32p))
        return out

    def rmsnorm(self, a, w):
        a = np.ascontiguousarray(a, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(a)
        self.lib.orc_rmsnorm(_ptr(a, _f32p), _ptr(w, _f32p), _ptr(out, _f32p), a.size)
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.orc_softmax(_ptr(x, _f32p), _ptr(out, _f32p), x.size)
        return out

    def swiglu(self, x, w_gate, w_up, w_down, f):
        x = np.ascontiguousarray(x, np.float32)
        gs = [np.ascontiguousarray(w, np.uint8) for w in (w_gate, w_up, w_down)]
        out = np.empty(x.size, np.float32)
        self.lib.orc_swiglu(_ptr(x, _f32p), *[_ptr(g, _u8p) for g in gs], _ptr(out, _f32p),
                            x.size, f)
        return out

    def rope_angles(self, base, pos, dim):
        out = np.empty(dim // 2, np.float32)
        self.lib.orc_rope_angles(float(base), pos, dim, _ptr(out, _f32p))
        return out

    def rope(self, q, k, thetas, dim):
        q = np.array(q, np.float32, copy=True)
        k = np.array(k, np.float32, copy=True)
        t = np.ascontiguousarray(thetas, np.float32)
        self.lib.orc_rope(_ptr(q, _f32p), q.size, _ptr(k, _f32p), k.size, _ptr(t, _f32p), dim)
        return q, k

    def embed(self, id_, table, dim):
        table = np.ascontiguousarray(table, np.uint8)
        out = np.empty(dim, np.float32)
        self.lib.orc_embed(id_, _ptr(table, _u8p), dim, _ptr(out, _f32p))
        return out

    def sample(self, logits):
        logits = np.ascontiguousarray(logits, np.float32)
        return self.lib.orc_sample(_ptr(logits, _f32p), logits.size)

    def set_threads(self, n):
        self.lib.orc_set_threads(int(n))

    def set_fast(self, on):
        """Eight rows per pass and parallel attention heads: the same bits, faster."""
        self.lib.orc_set_fast(1 if on else 0)

    def get_threads(self):
        return self.lib.orc_get_threads()

    # ---- model level -------------------------------------------------------
    def model(self, gguf, mode=0):
        """Binds a parsed GGUF (``oracle.gguf_ref.GGUF``) for forward passes."""
        return OracleModel(self, gguf, mode)


class OracleModel:
    """Holds the tensor table and a Cache; mirrors the reference's call pattern
    (``forward`` per token with an explicit ``pos``)."""

    LAYER_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                   "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")

    def __init__(self, orc, gguf, mode=0):
        self.orc = orc
        t = gguf.transformer()
        self.dims = Dims(
            n_layers=t["layers"], embed_dim=t["embed_dim"], head_dim=t["dim"],
            q_heads=t["q_heads"], kv_heads=t["k_v_heads"],
            ffn_dim=gguf.tensor_shape("blk.0.ffn_gate.weight")[1],
            vocab=gguf.tensor_shape("output.weight")[1],
            base_freq=t["base_freq"], mode=mode)
        names = ["token_embd.weight", "output_norm.weight", "output.weight"]
        for l in range(t["layers"]):
            names += [f"blk.{l}.{n}.weight" for n in self.LAYER_NAMES]
        self._arrays = [gguf.tensor_bytes(n) for n in names]  # keep alive
        self._table = (C.c_void_p * len(names))(
            *[a.ctypes.data_as(C.c_void_p).value for a in self._arrays])
        self.cache = orc.lib.orc_cache_new()

    def __del__(self):
        try:
            self.orc.lib.orc_cache_free(self.cache)
        except Exception:
            pass

    def reset(self):
        self.orc.lib.orc_cache_free(self.cache)
        self.cache = self.orc.lib.orc_cache_new()

    def embed(self, id_):
        return self.orc.embed(id_, self._arrays[0], self.dims.embed_dim)

    def forward_attn(self, token, pos):
        """forward with the per-layer dump, plus each layer's attention output
        (the output projection's input): (logits, dump, attn [L][H])."""
        attn = np.empty((self.dims.n_layers, self.dims.embed_dim), np.float32)
        self.orc.lib.orc_set_attn_dump(attn.ctypes.data)
        try:
            logits, dump = self.forward(token, pos, dump=True)
        finally:
            self.orc.lib.orc_set_attn_dump(None)
        return logits, dump, attn

    def forward(self, token, pos, dump=False):
        d = self.dims
        token = np.ascontiguousarray(token, np.float32)
        angles = self.orc.rope_angles(d.base_freq, pos, d.head_dim)
        logits = np.empty(d.vocab, np.float32)
        dump_arr = np.empty((d.n_layers + 1, d.embed_dim), np.float32) if dump else None
        rc = self.orc.lib.orc_forward(
            C.byref(d), self._table, self.cache, _ptr(token, _f32p), pos, _ptr(angles, _f32p),
            _ptr(logits, _f32p), _ptr(dump_arr, _f32p) if dump else None)
        if rc != 0:
            raise ValueError(f"oracle forward failed at pos {pos} (cache out of step)")
        return (logits, dump_arr) if dump else logits

    def generate_capped(self, prompt, cap):
        d = self.dims
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(cap, np.int32)
        last = np.zeros(d.vocab, np.float32)
        rc = self.orc.lib.orc_generate_capped(C.byref(d), self._table, _ptr(prompt, _i32p),
                                              prompt.size, cap, _ptr(out, _i32p),
                                              _ptr(last, _f32p))
        if rc != 0:
            raise ValueError("oracle generate_capped failed")
        return out, last


_INSTANCE = None


def load_oracle():
    global _INSTANCE
    if _INSTANCE is None:
        _INSTANCE = Oracle()
    return _INSTANCE
