"""Python binding of ``libtir.so`` (include/tir.h) -- the B200 decode runtime
for the Q8_0 Llama-2 path of ZeroR0R/tensor-inference-runtime.

Mirrors the reference's public surface:

* ``GGUF`` -- ``read_gguf`` + ``load_model``'s parse (src/reader.rs, src/lib.rs);
* ``Model`` -- the weights, uploaded once to HBM (``load_model``);
* ``State`` -- the KV cache (``Cache``, src/data.rs) plus ``forward``,
  ``forward_embedded``, ``generate_capped``, ``test_forward``;
* op functions (``q8_matmul``, ``rmsnorm``, ``softmax``, ``rope``, ...) taking
  device pointers (ints) or CUDA torch tensors.

The library is the only compute path: if ``libtir.so`` is missing or a call
fails, an exception is raised -- there is no CPU fallback.
"""
import ctypes as C
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libtir.so")

# tir_status (include/tir.h)
STATUS = {
    0: "OK", 1: "UNEXPECTED_EOF", 2: "INVALID_UTF8", 3: "BAD_MAGIC", 4: "BAD_VERSION",
    5: "UNSUPPORTED_TYPE", 6: "UNSUPPORTED_DTYPE", 7: "BAD_QUANT_BLOCK", 8: "MISSING_FIELD",
    9: "WRONG_TYPE", 10: "TENSOR_DATA", 11: "TENSOR_LOAD", 12: "BAD_TOKEN", 13: "IO",
    20: "CUDA", 21: "OOM", 22: "CTX_OVERFLOW", 23: "INVALID_ARG", 24: "UNSUPPORTED_SHAPE",
    25: "TIMEOUT", 26: "NO_DEVICE",
}
GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, \
    GGUF_STRING, GGUF_ARRAY, GGUF_U64, GGUF_I64, GGUF_F64 = range(13)


class TirError(RuntimeError):
    def __init__(self, status, message):
        self.status = status
        self.name = STATUS.get(status, str(status))
        self.message = message
        super().__init__(f"{self.name}: {message}")


class MetadataField(C.Structure):
    _fields_ = [("name", C.c_char_p), ("vtype", C.c_uint32), ("u", C.c_uint64), ("i", C.c_int64),
                ("f", C.c_double), ("str", C.c_void_p), ("str_len", C.c_uint64),
                ("array_type", C.c_uint32), ("array_len", C.c_uint64)]


class TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("shape", C.c_uint64 * 8),
                ("dtype", C.c_uint32), ("offset", C.c_uint64), ("data_bytes", C.c_uint64)]


class Transformer(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("dim", C.c_uint64), ("embed_dim", C.c_uint64),
                ("q_heads", C.c_uint64), ("k_v_heads", C.c_uint64), ("base_freq", C.c_float),
                ("mode", C.c_int32), ("kv_dim", C.c_uint64), ("ffn_dim", C.c_uint64),
                ("vocab", C.c_uint64)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


_vp, _u8p, _f32p, _i32p = C.c_void_p, C.POINTER(C.c_uint8), C.POINTER(C.c_float), C.POINTER(C.c_int32)
_i64, _sz = C.c_int64, C.c_size_t

# name -> (restype, argtypes); every function include/tir.h declares.
SIGNATURES = {
    "tir_last_error": (C.c_char_p, []),
    "tir_version": (C.c_char_p, []),
    "tir_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "tir_tokenizer_create": (C.c_int, [_vp, C.POINTER(_vp)]),
    "tir_tokenizer_create_from": (C.c_int, [C.POINTER(C.c_char_p), C.POINTER(C.c_uint64), _i64,
                                            C.POINTER(C.c_char_p), C.POINTER(C.c_uint64), _i64, C.POINTER(_vp)]),
    "tir_tokenizer_destroy": (None, [_vp]),
    "tir_tokenizer_vocab_size": (_i64, [_vp]),
    "tir_encode": (C.c_int, [_vp, C.c_char_p, _i64, _i32p, _i64, C.POINTER(_i64)]),
    "tir_decode": (C.c_int, [_vp, _i32p, _i64, C.c_char_p, _i64, C.POINTER(_i64)]),
    "tir_generate_capped_text": (C.c_int, [_vp, _vp, C.c_char_p, _i64, C.c_int32, _i32p]),
    "tir_generate_text": (C.c_int, [_vp, _vp, C.c_char_p, _i64, C.c_int32, C.c_char_p, _i64, C.POINTER(_i64),
                                    C.POINTER(C.c_int32)]),
    "tir_gguf_open_bytes": (C.c_int, [_vp, _sz, C.POINTER(_vp)]),
    "tir_gguf_close": (None, [_vp]),
    "tir_gguf_parse_general": (C.c_int, [_vp, _sz, _sz, C.c_uint64, C.POINTER(_vp), C.POINTER(_sz)]),
    "tir_gguf_parse_q8": (C.c_int, [C.c_uint64, _sz, _sz, _sz, C.POINTER(_sz)]),
    "tir_gguf_version": (C.c_uint32, [_vp]),
    "tir_gguf_n_metadata": (_i64, [_vp]),
    "tir_gguf_metadata": (C.c_int, [_vp, _i64, C.POINTER(MetadataField)]),
    "tir_gguf_metadata_item": (C.c_int, [_vp, _i64, C.c_uint64, C.POINTER(MetadataField)]),
    "tir_gguf_n_tensors": (_i64, [_vp]),
    "tir_gguf_tensor_info": (C.c_int, [_vp, _i64, C.POINTER(TensorInfo)]),
    "tir_gguf_tensor_data": (C.c_int, [_vp, C.c_char_p, C.POINTER(_vp), C.POINTER(_sz)]),
    "tir_gguf_transformer": (C.c_int, [_vp, C.POINTER(Transformer)]),
    "tir_model_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "tir_model_load_gguf": (C.c_int, [_vp, C.c_int, C.POINTER(_vp)]),
    "tir_model_info": (C.c_int, [_vp, C.POINTER(Transformer)]),
    "tir_model_set_mode": (C.c_int, [_vp, C.c_int32]),
    "tir_model_weight_bytes": (C.c_uint64, [_vp]),
    "tir_model_destroy": (None, [_vp]),
    "tir_state_create": (C.c_int, [_vp, C.c_int32, C.POINTER(_vp)]),
    "tir_state_reset": (C.c_int, [_vp]),
    "tir_state_len": (C.c_int32, [_vp]),
    "tir_state_stream": (_vp, [_vp]),
    "tir_state_destroy": (None, [_vp]),
    "tir_state_sync": (C.c_int, [_vp]),
    "tir_forward_embedded": (C.c_int, [_vp, _f32p, C.c_int32, _f32p]),
    "tir_forward": (C.c_int, [_vp, C.c_int32, C.c_int32, _f32p]),
    "tir_generate_capped": (C.c_int, [_vp, _i32p, C.c_int32, C.c_int32, _i32p, _f32p]),
    "tir_generate_capped_device": (C.c_int, [_vp, _vp, C.c_int32, C.c_int32, _vp]),
    "tir_test_forward": (C.c_int, [_vp, _i32p]),
    "tir_state_enable_dump": (C.c_int, [_vp, C.c_int32]),
    "tir_state_dump": (C.c_int, [_vp, _f32p]),
    "tir_debug_dump_layers": (C.c_int, [_vp, _f32p]),
    "tir_debug_dump_qact": (C.c_int, [_vp, _vp]),
    "tir_prefill": (C.c_int, [_vp, _vp, C.c_int32, C.c_int32, _vp]),
    "tir_state_enable_trace": (C.c_int, [_vp, C.c_int32]),
    "tir_state_trace_dims": (C.c_int, [_vp, _i32p, _i32p]),
    "tir_state_trace": (C.c_int, [_vp, C.POINTER(C.c_uint64)]),
    "tir_q8_scale_stride": (_i64, [_i64]),
    "tir_q8_repack": (C.c_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "tir_q8_matmul": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_q8_matmul_qact": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_q8_dequant": (C.c_int, [_vp, _i64, _vp, _vp]),
    "tir_embed": (C.c_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "tir_rmsnorm": (C.c_int, [_vp, _vp, _vp, _i64, _vp]),
    "tir_softmax": (C.c_int, [_vp, _vp, _i64, _vp]),
    "tir_rope": (C.c_int, [_vp, _i64, _vp, _i64, _f32p, _i64, _vp]),
    "tir_rope_angles": (None, [C.c_float, _i64, _i64, _f32p]),
    "tir_swiglu": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_swiglu_static": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_batch_create": (C.c_int, [_vp, C.c_int32, C.c_int32, C.c_int32, C.POINTER(_vp)]),
    "tir_batch_create_paged": (C.c_int, [_vp, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.POINTER(_vp)]),
    "tir_batch_reset_seq": (C.c_int, [_vp, C.c_int32]),
    "tir_batch_seq_len": (C.c_int32, [_vp, C.c_int32]),
    "tir_batch_free_pages": (C.c_int32, [_vp]),
    "tir_batch_step_ragged": (C.c_int, [_vp, _vp, _vp, _vp]),
    "tir_batch_destroy": (None, [_vp]),
    "tir_batch_reset": (C.c_int, [_vp]),
    "tir_batch_len": (C.c_int32, [_vp]),
    "tir_batch_stream": (_vp, [_vp]),
    "tir_batch_step": (C.c_int, [_vp, _vp, C.c_int32, _vp]),
    "tir_batch_generate": (C.c_int, [_vp, _vp, C.c_int32, C.c_int32, _vp]),
    "tir_batch_logits": (C.c_int, [_vp, _vp]),
    "tir_batch_dump_rows": (C.c_int, [_vp, _vp, C.c_int32]),
    "tir_batch_dump": (C.c_int, [_vp, _vp]),
    "tir_q8_gemm_bytes": (_i64, [_i64, _i64]),
    "tir_q8_gemm_rows": (_i64, [_i64]),
    "tir_q8_gemm_prepare": (C.c_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "tir_q8_matmul_batch": (C.c_int, [_vp, _i64, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_q8_tile_rows": (_i64, [_i64]),
    "tir_q8_tiled_bytes": (_i64, [_i64, _i64]),
    "tir_q8_repack_tiled": (C.c_int, [_vp, _i64, _i64, _vp, _vp]),
    "tir_q8_matmul_tiled": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_activated_q8": (C.c_int, [_vp, _i64, _vp, _vp]),
    "tir_q8_act_matmul": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "tir_argmax": (C.c_int, [_vp, _i64, _vp, _vp]),
    "tir_attention": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "tir_ops_check": (C.c_int, [_vp]),
    "tir_debug_fail_alloc_after": (None, [_i64]),
    "tir_debug_alloc_count": (_i64, []),
    "tir_debug_hold_phase": (C.c_int, [_vp, C.c_int32, C.c_int32]),
    "tir_debug_hold_next_op": (C.c_int, [C.c_int32]),
}

_lib = None
def lib():
    """Loads libtir.so (built in-tree by tir.build); raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with tir.build.build() "
                              "(the CUDA library is the only implementation)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status != 0:
        raise TirError(status, lib().tir_last_error().decode(errors="replace"))


def _ptr(x):
    """Device pointer of a CUDA torch tensor, or an int address."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:
            return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def version():
    return lib().tir_version().decode()


# ---------------------------------------------------------------------------
# GGUF
# ---------------------------------------------------------------------------
class GGUF:
    """read_gguf + load_model's parse (src/reader.rs:15, src/lib.rs:29-138)."""

    def __init__(self, handle):
        self._h = C.c_void_p(handle)
        self._destroy = lib().tir_gguf_close  # held by the object: usable at interpreter teardown

    @classmethod
    def open(cls, path):
        h = C.c_void_p()
        check(lib().tir_gguf_open(os.fsencode(path), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_bytes(cls, data):
        buf = C.create_string_buffer(bytes(data), len(data))
        h = C.c_void_p()
        check(lib().tir_gguf_open_bytes(C.cast(buf, C.c_void_p), len(data), C.byref(h)))
        return cls(h.value)

    @staticmethod
    def parse_general(data, offset, count):
        """parse_general (src/reader.rs:98-169): ([(name, vtype, value)], end)."""
        buf = C.create_string_buffer(bytes(data), max(1, len(data)))
        h = C.c_void_p()
        end = C.c_size_t()
        check(lib().tir_gguf_parse_general(C.cast(buf, C.c_void_p), len(data), offset, count,
                                           C.byref(h), C.byref(end)))
        g = GGUF(h.value)
        try:
            return g.metadata(), end.value
        finally:
            g.close()

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            self._destroy(h)

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def version(self):
        return lib().tir_gguf_version(self._h)

    @staticmethod
    def _value(f, items=None):
        if f.vtype == GGUF_STRING:
            return C.string_at(f.str, f.str_len).decode()
        if f.vtype == GGUF_ARRAY:
            return (f.array_type, items)
        if f.vtype in (GGUF_U8, GGUF_U16, GGUF_U32, GGUF_U64):
            return f.u
        if f.vtype == GGUF_BOOL:
            return bool(f.u)
        if f.vtype in (GGUF_I8, GGUF_I16, GGUF_I32, GGUF_I64):
            return f.i
        return f.f

    def metadata(self):
        out = []
        for i in range(lib().tir_gguf_n_metadata(self._h)):
            f = MetadataField()
            check(lib().tir_gguf_metadata(self._h, i, C.byref(f)))
            items = None
            if f.vtype == GGUF_ARRAY:
                items = []
                for j in range(f.array_len):
                    it = MetadataField()
                    check(lib().tir_gguf_metadata_item(self._h, i, j, C.byref(it)))
                    items.append(self._value(it))
            out.append((f.name.decode(), f.vtype, self._value(f, items)))
        return out

    def tensors(self):
        out = []
        for i in range(lib().tir_gguf_n_tensors(self._h)):
            t = TensorInfo()
            check(lib().tir_gguf_tensor_info(self._h, i, C.byref(t)))
            out.append({"name": t.name.decode(), "n_elements": t.n_dims,
                        "shape": [t.shape[d] for d in range(t.n_dims)], "dtype": t.dtype,
                        "offset": t.offset, "data_bytes": t.data_bytes})
        return out

    def tensor_bytes(self, name):
        p = C.c_void_p()
        n = C.c_size_t()
        check(lib().tir_gguf_tensor_data(self._h, name.encode(), C.byref(p), C.byref(n)))
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value,)).copy()

    def transformer(self):
        t = Transformer()
        check(lib().tir_gguf_transformer(self._h, C.byref(t)))
        return t.as_dict()


def parse_q8(count, byte_count, map_len, offset):
    """parse_q8 (src/reader.rs:258-272): byte length of the tensor data."""
    n = C.c_size_t()
    check(lib().tir_gguf_parse_q8(count, byte_count, map_len, offset, C.byref(n)))
    return n.value


# ---------------------------------------------------------------------------
# Model / State
# ---------------------------------------------------------------------------
class Tokenizer:
    """BPE encode / decode (src/tokenizer.rs:37-150) over a vocab and merge list."""

    def __init__(self, handle):
        self._h = handle
        self._destroy = lib().tir_tokenizer_destroy  # held by the object: usable at interpreter teardown

    @classmethod
    def from_gguf(cls, gguf):
        h = _vp()
        check(lib().tir_tokenizer_create(gguf.handle, C.byref(h)))
        return cls(h)

    @classmethod
    def from_lists(cls, tokens, merges):
        tb = [t.encode("utf-8") for t in tokens]
        mb = [m.encode("utf-8") for m in merges]
        tp = (C.c_char_p * max(len(tb), 1))(*tb)
        tl = (C.c_uint64 * max(len(tb), 1))(*[len(b) for b in tb])
        mp = (C.c_char_p * max(len(mb), 1))(*mb)
        ml = (C.c_uint64 * max(len(mb), 1))(*[len(b) for b in mb])
        h = _vp()
        check(lib().tir_tokenizer_create_from(tp, tl, len(tb), mp, ml, len(mb), C.byref(h)))
        return cls(h)

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            self._destroy(h)

    def __del__(self):
        self.close()

    @property
    def handle(self):
        return self._h

    def __len__(self):
        return int(lib().tir_tokenizer_vocab_size(self._h))

    def encode(self, text):
        raw = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        n = _i64()
        check(lib().tir_encode(self._h, raw, len(raw), None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        check(lib().tir_encode(self._h, raw, len(raw), out.ctypes.data_as(_i32p), n.value, C.byref(n)))
        return out[:n.value]

    def decode(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        n = _i64()
        check(lib().tir_decode(self._h, ids.ctypes.data_as(_i32p), ids.size, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        check(lib().tir_decode(self._h, ids.ctypes.data_as(_i32p), ids.size, buf, n.value + 1, C.byref(n)))
        return buf.raw[:n.value].decode("utf-8")


class Model:
    """Weights resident in HBM (load_model, src/lib.rs:29-138)."""

    def __init__(self, path=None, device=0, gguf=None):
        h = C.c_void_p()
        if gguf is not None:
            check(lib().tir_model_load_gguf(gguf.handle, device, C.byref(h)))
        else:
            check(lib().tir_model_load(os.fsencode(path), device, C.byref(h)))
        self._h = h
        self._destroy = lib().tir_model_destroy  # held by the object: usable at interpreter teardown
        self.device = device
        t = Transformer()
        check(lib().tir_model_info(self._h, C.byref(t)))
        self.info = t.as_dict()

    @property
    def handle(self):
        return self._h

    def weight_bytes(self):
        return lib().tir_model_weight_bytes(self._h)

    def set_mode(self, mode):
        check(lib().tir_model_set_mode(self._h, mode))

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            self._destroy(h)

    def __del__(self):
        self.close()

    def state(self, max_ctx=2048):
        return State(self, max_ctx)


class State:
    """The KV cache of one sequence (Cache, src/data.rs:41-51) and its drivers."""

    def __init__(self, model, max_ctx=2048):
        self.model = model
        h = C.c_void_p()
        check(lib().tir_state_create(model.handle, max_ctx, C.byref(h)))
        self._h = h
        self._destroy = lib().tir_state_destroy  # held by the object: usable at interpreter teardown
        self.max_ctx = max_ctx
        self.vocab = model.info["vocab"]
        self.embed_dim = model.info["embed_dim"]
        self.layers = model.info["layers"]

    @property
    def handle(self):
        return self._h

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            self._destroy(h)

    def __del__(self):
        self.close()

    def reset(self):
        check(lib().tir_state_reset(self._h))

    def __len__(self):
        return lib().tir_state_len(self._h)

    def stream(self):
        return lib().tir_state_stream(self._h)

    def sync(self):
        check(lib().tir_state_sync(self._h))

    def forward_embedded(self, x, pos):
        """forward (src/forward.rs:13-258) on an embedded input; returns logits."""
        x = np.ascontiguousarray(x, np.float32)
        logits = np.empty(self.vocab, np.float32)
        check(lib().tir_forward_embedded(self._h, x.ctypes.data_as(_f32p), pos,
                                         logits.ctypes.data_as(_f32p)))
        return logits

    def forward(self, token_id, pos):
        """embed + forward: token id in, logits out."""
        logits = np.empty(self.vocab, np.float32)
        check(lib().tir_forward(self._h, int(token_id), pos, logits.ctypes.data_as(_f32p)))
        return logits

    def generate_capped(self, prompt, cap, want_logits=False):
        """generate_capped (src/lib.rs:239-314) on token ids."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(cap, 1), np.int32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib().tir_generate_capped(self._h, prompt.ctypes.data_as(_i32p), prompt.size, cap,
                                        out.ctypes.data_as(_i32p),
                                        logits.ctypes.data_as(_f32p) if want_logits else None))
        return (out[:cap], logits) if want_logits else out[:cap]

    def generate_capped_text(self, tokenizer, text, cap):
        """generate_capped (src/lib.rs:239-314) on text."""
        raw = text.encode("utf-8")
        out = np.zeros(max(cap, 1), np.int32)
        check(lib().tir_generate_capped_text(self._h, tokenizer.handle, raw, len(raw), cap,
                                             out.ctypes.data_as(_i32p)))
        return out[:cap]

    def generate_text(self, tokenizer, text, max_new):
        """generate (src/lib.rs:140-236): greedy until id 13 or 2, at most max_new ids.
        Returns (text, number of ids kept)."""
        raw = text.encode("utf-8")
        n, k = _i64(), C.c_int32()
        cap = 64 * max(max_new, 1) + 1
        buf = C.create_string_buffer(cap)
        check(lib().tir_generate_text(self._h, tokenizer.handle, raw, len(raw), max_new, buf, cap,
                                      C.byref(n), C.byref(k)))
        return buf.raw[:min(n.value, cap - 1)].decode("utf-8"), k.value

    def prefill(self, ids, want_logits=True):
        """The prompt pass alone (positions 0..len-1 of an empty cache); the last
        position's logits, or None."""
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib().tir_prefill(self._h, ids.ctypes.data, 1, len(ids),
                                logits.ctypes.data if want_logits else None))
        return logits

    def generate_capped_device(self, prompt_dev, n_prompt, cap, out_dev):
        check(lib().tir_generate_capped_device(self._h, _ptr(prompt_dev), n_prompt, cap,
                                               _ptr(out_dev)))

    def test_forward(self):
        """test_forward (src/lib.rs:316-328)."""
        out = C.c_int32()
        check(lib().tir_test_forward(self._h, C.byref(out)))
        return out.value

    def enable_dump(self, on=True):
        check(lib().tir_state_enable_dump(self._h, 1 if on else 0))

    def dump_qact(self):
        """Mode::Quantize: [(2 L + 1), embed_dim / 32, 34] uint8 Q8_0 blocks of the
        last forward's quantised inputs (q|k|v of layer l at 2 l, o at 2 l + 1,
        lm_head at 2 L)."""
        nb = self.embed_dim // 32
        out = np.empty((2 * self.layers + 1, nb, 34), np.uint8)
        check(lib().tir_debug_dump_qact(self._h, out.ctypes.data))
        return out

    def enable_trace(self, step):
        check(lib().tir_state_enable_trace(self._h, int(step)))

    def hold_phase(self, phase, timeout_us):
        """Test hook: the next launch's wait at `phase` is never met and runs
        out after timeout_us (the launch then returns TIR_ERR_TIMEOUT)."""
        check(lib().tir_debug_hold_phase(self._h, int(phase), int(timeout_us)))

    def trace(self):
        """[n_phases, grid, 8]: stamps (ns) start/ready/staged/released, ns waiting
        for ring data, tiles, ns waiting for the previous phase."""
        n, g = C.c_int32(), C.c_int32()
        check(lib().tir_state_trace_dims(self._h, C.byref(n), C.byref(g)))
        out = np.zeros((n.value, g.value, 8), np.uint64)
        check(lib().tir_state_trace(self._h, out.ctypes.data_as(C.POINTER(C.c_uint64))))
        return out

    def dump(self):
        out = np.empty((self.layers + 1, self.embed_dim), np.float32)
        check(lib().tir_state_dump(self._h, out.ctypes.data_as(_f32p)))
        return out

    def dump_layers(self):
        """[layers, embed_dim]: every layer's output in the last forward."""
        out = np.empty((self.layers, self.embed_dim), np.float32)
        check(lib().tir_debug_dump_layers(self._h, out.ctypes.data_as(_f32p)))
        return out


# ---------------------------------------------------------------------------
# op level (device pointers)
# ---------------------------------------------------------------------------
def q8_scale_stride(k):
    return lib().tir_q8_scale_stride(k)


def q8_repack(blocks, rows, k, quants, scales, stream=None):
    check(lib().tir_q8_repack(_ptr(blocks), rows, k, _ptr(quants), _ptr(scales), _stream(stream)))


def q8_matmul(x, quants, scales, out, n, k, stream=None):
    check(lib().tir_q8_matmul(_ptr(x), _ptr(quants), _ptr(scales), _ptr(out), n, k, _stream(stream)))


def q8_matmul_qact(x, quants, scales, out, n, k, stream=None):
    """matmul in Mode::Quantize (src/forward.rs:266-273) from an f32 input."""
    check(lib().tir_q8_matmul_qact(_ptr(x), _ptr(quants), _ptr(scales), _ptr(out), n, k, _stream(stream)))


class Batch:
    """n_seqs sequences on the tensor-core path with a paged KV cache (pool of
    n_pages pages of 16 positions; default: every sequence can reach max_ctx)."""

    def __init__(self, model, n_seqs, max_ctx, max_tokens_per_seq, n_pages=None):
        self.model = model
        self.n_seqs = n_seqs
        self.vocab = model.info["vocab"]
        h = C.c_void_p()
        if n_pages is None:
            check(lib().tir_batch_create(model.handle, n_seqs, max_ctx, max_tokens_per_seq, C.byref(h)))
        else:
            check(lib().tir_batch_create_paged(model.handle, n_seqs, max_ctx, max_tokens_per_seq, n_pages,
                                               C.byref(h)))
        self._h = h
        self._destroy = lib().tir_batch_destroy  # held by the object: usable at interpreter teardown

    @property
    def handle(self):
        return self._h

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            self._destroy(h)

    def __del__(self):
        self.close()

    def reset(self):
        check(lib().tir_batch_reset(self._h))

    def reset_seq(self, seq):
        check(lib().tir_batch_reset_seq(self._h, seq))

    def seq_len(self, seq):
        return lib().tir_batch_seq_len(self._h, seq)

    def free_pages(self):
        return lib().tir_batch_free_pages(self._h)

    def step_ragged(self, ids_per_seq):
        """ids_per_seq: one id sequence per batch sequence (empty: idle) ->
        greedy next id per sequence (meaningless for idle ones)."""
        counts = np.array([len(x) for x in ids_per_seq], np.int32)
        assert counts.size == self.n_seqs
        flat = np.ascontiguousarray(np.concatenate([np.asarray(x, np.int32).reshape(-1) for x in ids_per_seq])
                                    if counts.sum() else np.zeros(1, np.int32), np.int32)
        out = np.zeros(self.n_seqs, np.int32)
        check(lib().tir_batch_step_ragged(self._h, flat.ctypes.data, counts.ctypes.data, out.ctypes.data))
        return out

    def __len__(self):
        return lib().tir_batch_len(self._h)

    def stream(self):
        return lib().tir_batch_stream(self._h)

    def step(self, ids):
        """ids [n_seqs][tokens_per_seq] -> greedy next id per sequence."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(self.n_seqs, -1)
        out = np.zeros(self.n_seqs, np.int32)
        check(lib().tir_batch_step(self._h, ids.ctypes.data, ids.shape[1], out.ctypes.data))
        return out

    def generate(self, prompts, cap):
        """prompts [n_seqs][n_prompt] -> ids [n_seqs][cap] (n_prompt + cap forwards each)."""
        prompts = np.ascontiguousarray(prompts, np.int32).reshape(self.n_seqs, -1)
        out = np.zeros((self.n_seqs, cap), np.int32)
        check(lib().tir_batch_generate(self._h, prompts.ctypes.data, prompts.shape[1], cap, out.ctypes.data))
        return out

    def logits(self):
        """[n_seqs, vocab]: each sequence's last-row logits of the last forward."""
        out = np.empty((self.n_seqs, self.vocab), np.float32)
        check(lib().tir_batch_logits(self._h, out.ctypes.data))
        return out

    def dump_rows(self, rows):
        """Arms the per-layer dump of step rows `rows` (sequence-major indices)
        for later forwards outside the decode graph (prefill, ragged steps)."""
        rows = np.ascontiguousarray(rows, np.int32)
        check(lib().tir_batch_dump_rows(self._h, rows.ctypes.data if rows.size else None, rows.size))
        self._dump_n = int(rows.size)

    def dump(self):
        """[n_rows, layers, embed_dim]: the armed rows' layer outputs of the last such forward."""
        out = np.empty((self._dump_n, self.model.info["layers"], self.model.info["embed_dim"]), np.float32)
        check(lib().tir_batch_dump(self._h, out.ctypes.data))
        return out


def q8_gemm_prepare(blocks, n, k, stream=None):
    """Tensor-core layout of a Q8_0 [n][k] matrix from device blocks: (w, w_pow2)."""
    import torch
    w = torch.empty(lib().tir_q8_gemm_bytes(n, k), dtype=torch.uint8, device=blocks.device)
    p2 = torch.empty(lib().tir_q8_gemm_rows(n), dtype=torch.float32, device=blocks.device)
    check(lib().tir_q8_gemm_prepare(_ptr(blocks), n, k, _ptr(w), _ptr(p2), _stream(stream)))
    return w, p2


def q8_matmul_batch(x, tokens, w, y, n, k, stream=None):
    """y[t][j] = sum_c x[t][c] W[j][c] on the tensor cores; w = (weights, pow2)."""
    check(lib().tir_q8_matmul_batch(_ptr(x), tokens, _ptr(w[0]), _ptr(w[1]), _ptr(y), n, k, _stream(stream)))


def q8_tile_rows(k):
    return lib().tir_q8_tile_rows(k)


def q8_tiled_bytes(n, k):
    return lib().tir_q8_tiled_bytes(n, k)


def q8_repack_tiled(blocks, rows, k, out, stream=None):
    check(lib().tir_q8_repack_tiled(_ptr(blocks), rows, k, _ptr(out), _stream(stream)))


def q8_matmul_tiled(x, w, out, n, k, stream=None):
    check(lib().tir_q8_matmul_tiled(_ptr(x), _ptr(w), _ptr(out), n, k, _stream(stream)))


def q8_dequant(blocks, n_blocks, out, stream=None):
    check(lib().tir_q8_dequant(_ptr(blocks), n_blocks, _ptr(out), _stream(stream)))


def embed(blocks, vocab, id_, dim, out, stream=None):
    check(lib().tir_embed(_ptr(blocks), vocab, id_, dim, _ptr(out), _stream(stream)))


def rmsnorm(x, w, out, n, stream=None):
    check(lib().tir_rmsnorm(_ptr(x), _ptr(w), _ptr(out), n, _stream(stream)))


def softmax(x, out, n, stream=None):
    check(lib().tir_softmax(_ptr(x), _ptr(out), n, _stream(stream)))


def rope_angles(base, pos, dim):
    out = np.empty(dim // 2, np.float32)
    lib().tir_rope_angles(float(base), pos, dim, out.ctypes.data_as(_f32p))
    return out


def rope(q, nq, k, nk, thetas, dim, stream=None):
    t = np.ascontiguousarray(thetas, np.float32)
    check(lib().tir_rope(_ptr(q), nq, _ptr(k), nk, t.ctypes.data_as(_f32p), dim, _stream(stream)))


def swiglu(x, gate, up, down, out, k, f, stream=None):
    """gate/up/down: (quants, scales) pairs of split-layout matrices."""
    check(lib().tir_swiglu(_ptr(x), _ptr(gate[0]), _ptr(gate[1]), _ptr(up[0]), _ptr(up[1]),
                           _ptr(down[0]), _ptr(down[1]), _ptr(out), k, f, _stream(stream)))


def swiglu_static(x, gate, up, down, out, k, f, stream=None):
    """swiglu with its intermediates in a fixed per-device array (f <= 6144);
    allocates no device memory.  Calls on one device must not overlap."""
    check(lib().tir_swiglu_static(_ptr(x), _ptr(gate[0]), _ptr(gate[1]), _ptr(up[0]), _ptr(up[1]),
                                  _ptr(down[0]), _ptr(down[1]), _ptr(out), k, f, _stream(stream)))


def ops_check(stream=None):
    """Synchronises `stream`; raises TirError(TIMEOUT) if an op launched on the
    current device since the last check had a device-side wait give up."""
    check(lib().tir_ops_check(_stream(stream)))


def fail_alloc_after(n):
    """Test hook: the n-th next allocation of the library fails once (n < 0: off)."""
    lib().tir_debug_fail_alloc_after(int(n))


def hold_next_op(timeout_us):
    """Test hook: the next streaming matvec runs a held second pass that gives
    up after timeout_us (reported by ops_check)."""
    check(lib().tir_debug_hold_next_op(int(timeout_us)))


def alloc_count():
    """Allocation calls the library has made so far (device, async, pinned)."""
    return int(lib().tir_debug_alloc_count())


def activated_q8(x, k, out_blocks, stream=None):
    check(lib().tir_activated_q8(_ptr(x), k, _ptr(out_blocks), _stream(stream)))


def q8_act_matmul(x_blocks, quants, scales, out, n, k, stream=None):
    check(lib().tir_q8_act_matmul(_ptr(x_blocks), _ptr(quants), _ptr(scales), _ptr(out), n, k,
                                  _stream(stream)))


def argmax(x, n, out_id, stream=None):
    check(lib().tir_argmax(_ptr(x), n, _ptr(out_id), _stream(stream)))


def attention(q, k_cache, v_cache, out, q_heads, k_v_heads, dim, n_ctx, max_ctx, stream=None):
    check(lib().tir_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), q_heads, k_v_heads,
                              dim, n_ctx, max_ctx, _stream(stream)))
