"""Python binding of libneedle_c.so — the B200 needle engine.

Mirrors the reference's Python-facing engine API (crates/needle-python/src/
lib.rs:5-92 wraps NeedleEngine::{load, run, run_stream, run_batch}) over the
C ABI in include/needle.h and include/needle_b200.h, with ctypes.  There is
no CPU fallback: every call goes through the CUDA library, and loading fails
loudly when it is missing.

Import it by path (the directory name is not a Python identifier):
    spec = importlib.util.spec_from_file_location("needle_b200", ".../needle-rs_b200/__init__.py")
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libneedle_c.so")

STOP_ON_EOS = 1
DEVICE_POINTERS = 2
NO_GRAPH = 4
NO_PDL = 8

_lib = None


class NeedleError(RuntimeError):
    pass


def build(force=False):
    import importlib.util

    spec = importlib.util.spec_from_file_location("needle_b200_build", os.path.join(HERE, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force)


def lib():
    """The loaded libneedle_c.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NeedleError(f"{LIB_PATH} is missing: run needle-rs_b200/build.py (nvcc, sm_100a)")
        L = C.CDLL(LIB_PATH)
        P, S, I, U32, I64 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_int64
        sig = {
            "needle_load": (P, [C.c_char_p, C.c_char_p]),
            "needle_load_bytes": (P, [P, S, P, S]),
            "needle_run": (P, [P, C.c_char_p, C.c_char_p]),
            "needle_run_stream": (P, [P, C.c_char_p, C.c_char_p, P, P]),
            "needle_contrastive_dim": (S, [P]),
            "needle_encode_contrastive": (C.c_bool, [P, C.c_char_p, P, S]),
            "needle_retrieve_tools": (S, [P, C.c_char_p, P, S, S, P, P]),
            "needle_free_str": (None, [P]),
            "needle_free": (None, [P]),
            "needle_last_error": (C.c_char_p, []),
            "needle_device_count": (I, []),
            "needle_load_on_device": (P, [C.c_char_p, C.c_char_p, I]),
            "needle_load_bytes_on_device": (P, [P, S, P, S, I]),
            "needle_model_config": (I, [P, P]),
            "needle_handle_device": (I, [P]),
            "needle_run_batch_ids": (I, [P, P, P, S, U32, P, U32, P, P]),
            "needle_run_batch_ids_logits": (I, [P, P, P, S, U32, P, U32, P, P, P]),
            "needle_batch_prepare": (P, [P, P, P, S, U32, P, U32]),
            "needle_batch_run": (I, [P]),
            "needle_batch_sync": (I, [P]),
            "needle_batch_results": (I, [P, P, P]),
            "needle_batch_stream": (P, [P]),
            "needle_batch_kernel_launches": (I64, [P]),
            "needle_batch_time_kernel": (I, [P, I]),
            "needle_batch_kernel_timing": (I, [P, P, P, P, P]),
            "needle_batch_free": (None, [P]),
            "needle_batch_begin": (I, [P]),
            "needle_batch_set_step_mask": (I, [P, U32, P]),
            "needle_batch_step": (I, [P, P, P, P]),
            "needle_shard_requests": (I, [P, S, I, P]),
            "needle_debug_forward": (I, [P, P, S, P, S, P, P]),
            "needle_int4_matmul": (I, [P, S, S, P, P, S, S, P, P]),
            "needle_int4_matmul_ex": (I, [P, S, S, P, P, S, S, P, U32, P]),
            "needle_int4_plan_create": (P, [P, P, S, S, S, S, P]),
            "needle_int4_plan_matmul": (I, [P, P, S, P, U32, P]),
            "needle_int4_plan_status": (I, [P]),
            "needle_int4_plan_free": (None, [P]),
            "needle_int4_quantize": (I, [P, S, S, P, P, P]),
            "needle_int4_dequantize": (I, [P, P, S, S, S, P, P]),
            "needle_run_batch": (I, [P, P, P, S, P]),
            "needle_vocab_parse": (P, [C.c_char_p, S]),
            "needle_handle_vocab": (P, [P]),
            "needle_vocab_size": (S, [P]),
            "needle_vocab_encode": (S, [P, C.c_char_p, P, S]),
            "needle_vocab_decode": (P, [P, P, S]),
            "needle_vocab_free": (None, [P]),
            "needle_snake_case": (P, [C.c_char_p]),
            "needle_tools_encoder_text": (P, [C.c_char_p]),
            "needle_tools_restore_names": (P, [C.c_char_p, C.c_char_p]),
            "needle_constraint_new": (P, [C.c_char_p, P]),
            "needle_constraint_update": (I, [P, U32]),
            "needle_constraint_feed": (I, [P, C.c_char_p, S]),
            "needle_constraint_mask": (I, [P, S, P]),
            "needle_constraint_state": (I, [P]),
            "needle_constraint_free": (None, [P]),
            "needle_ffn_forward": (I, [P, S, S, S, P, P, P, P, P, P, I, P, P]),
            "needle_ffn_forward_noalloc": (I, [P, S, S, S, P, P, P, P, P, P, I, P, P]),
            "needle_hbm_read_gbs": (I, [S, I, P]),
            "needle_ffn_plan_create": (P, [S, S, P, P, P, P, P, P, S, P]),
            "needle_ffn_plan_forward": (I, [P, P, S, I, P, P]),
            "needle_ffn_plan_status": (I, [P]),
            "needle_ffn_plan_free": (None, [P]),
            "needle_safetensors_parse": (P, [P, S]),
            "needle_safetensors_metadata": (C.c_char_p, [P, C.c_char_p]),
            "needle_safetensors_get_f32": (S, [P, C.c_char_p, P, S]),
            "needle_safetensors_free": (None, [P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    e = lib().needle_last_error()
    return e.decode() if e else None


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _check(rc):
    if rc != 0:
        raise NeedleError(last_error() or "needle call failed")


def device_count():
    return lib().needle_device_count()


CONFIG_KEYS = ["d_model", "num_heads", "num_kv_heads", "num_layers", "num_dec_layers", "vocab_size",
               "max_enc_len", "max_dec_len", "ffn_dim", "no_feedforward", "activation", "head_dim"]


def _csr(prompts):
    lens = np.array([len(p) for p in prompts], np.uint64)
    off = np.zeros(len(prompts) + 1, np.uint64)
    np.cumsum(lens, out=off[1:])
    ids = np.concatenate([np.asarray(p, np.uint32) for p in prompts]) if prompts else np.zeros(0, np.uint32)
    return np.ascontiguousarray(ids, np.uint32), off


class NeedleEngine:
    """A model loaded on one GPU (NeedleEngine of crates/needle-infer/src/engine.rs)."""

    def __init__(self, handle):
        self._h = handle
        cfg = np.zeros(12, np.int64)
        _check(lib().needle_model_config(self._h, _p(cfg)))
        self.cfg = dict(zip(CONFIG_KEYS, (int(v) for v in cfg)))
        self.device = lib().needle_handle_device(self._h)

    @classmethod
    def load(cls, weights_path, vocab_path, device=None):
        L = lib()
        if device is None:
            h = L.needle_load(str(weights_path).encode(), str(vocab_path).encode())
        else:
            h = L.needle_load_on_device(str(weights_path).encode(), str(vocab_path).encode(), int(device))
        if not h:
            raise NeedleError(last_error() or "load failed")
        return cls(h)

    @classmethod
    def from_bytes(cls, weights, vocab_text, device=None):
        w = np.frombuffer(bytes(weights), np.uint8)
        v = np.frombuffer(vocab_text.encode() if isinstance(vocab_text, str) else bytes(vocab_text), np.uint8)
        vp = _p(v) if v.size else C.c_void_p(C.addressof(C.c_char()))
        if device is None:
            h = lib().needle_load_bytes(_p(w), w.size, vp, v.size)
        else:
            h = lib().needle_load_bytes_on_device(_p(w), w.size, vp, v.size, int(device))
        if not h:
            raise NeedleError(last_error() or "load failed")
        return cls(h)

    def close(self):
        if getattr(self, "_h", None):
            lib().needle_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ── text level (needle_run / needle_run_stream) ──
    def run(self, query, tools_json):
        r = lib().needle_run(self._h, query.encode(), tools_json.encode())
        if not r:
            raise NeedleError(last_error() or "needle_run failed")
        s = C.string_at(r).decode()
        lib().needle_free_str(r)
        return s

    def run_batch(self, queries, tools_jsons):
        """NeedleEngine::run_batch: one output string per (query, tools) pair."""
        n = len(queries)
        if len(tools_jsons) != n:
            raise ValueError("queries and tools_jsons differ in length")
        qa = (C.c_char_p * max(n, 1))(*[q.encode() for q in queries])
        ta = (C.c_char_p * max(n, 1))(*[t.encode() for t in tools_jsons])
        out = (C.c_void_p * max(n, 1))()
        _check(lib().needle_run_batch(self._h, qa, ta, n, out))
        res = []
        for i in range(n):
            res.append(C.string_at(out[i]).decode())
            lib().needle_free_str(out[i])
        return res

    @property
    def contrastive_dim(self):
        return lib().needle_contrastive_dim(self._h)

    def encode_contrastive(self, text):
        """L2-normalised contrastive embedding, or None without a head."""
        c = self.contrastive_dim
        if not c:
            return None
        out = np.zeros(c, np.float32)
        if not lib().needle_encode_contrastive(self._h, text.encode(), _p(out), c):
            raise NeedleError(last_error() or "needle_encode_contrastive failed")
        return out

    def retrieve_tools(self, query, tool_descriptions, top_k):
        """[(index, score)] by descending contrastive similarity (retrieve_tools)."""
        n = len(tool_descriptions)
        descs = (C.c_char_p * max(n, 1))(*[t.encode() for t in tool_descriptions])
        idx = np.zeros(max(top_k, 1), np.uint64)
        sc = np.zeros(max(top_k, 1), np.float32)
        m = lib().needle_retrieve_tools(self._h, query.encode(), descs, n, top_k, _p(idx), _p(sc))
        return [(int(idx[i]), float(sc[i])) for i in range(m)]

    def vocab(self):
        """The handle's vocabulary (valid while the engine is open)."""
        return Vocab(_handle=lib().needle_handle_vocab(self._h), _owner=self)

    def run_stream(self, query, tools_json, on_token):
        CB = C.CFUNCTYPE(None, C.c_uint32, C.c_char_p, C.c_void_p)
        cb = CB(lambda tid, piece, ud: on_token(int(tid), piece.decode()))
        r = lib().needle_run_stream(self._h, query.encode(), tools_json.encode(), C.cast(cb, C.c_void_p), None)
        if not r:
            raise NeedleError(last_error() or "needle_run_stream failed")
        s = C.string_at(r).decode()
        lib().needle_free_str(r)
        return s

    # ── token-ID level ──
    def run_batch_ids(self, prompts, max_new, mask_bits=None, stop_on_eos=False, want_logits=False, graph=True,
                      pdl=True):
        """Greedy generation for a list of prompts (lists of token ids).

        mask_bits: None or uint64 [n_req, max_new, ceil(V/64)].  Returns
        (ids [n_req, max_new] uint32, lens [n_req] uint32[, logits])."""
        ids, off = _csr(prompts)
        n = len(prompts)
        out = np.zeros((n, max_new), np.uint32)
        lens = np.zeros(n, np.uint32)
        mb = None if mask_bits is None else np.ascontiguousarray(mask_bits, np.uint64)
        flags = (STOP_ON_EOS if stop_on_eos else 0) | (0 if graph else NO_GRAPH) | (0 if pdl else NO_PDL)
        if want_logits:
            lg = np.zeros((n, max_new, self.cfg["vocab_size"]), np.float32)
            _check(lib().needle_run_batch_ids_logits(self._h, _p(ids), _p(off), n, max_new, _p(mb), flags,
                                                     _p(out), _p(lens), _p(lg)))
            return out, lens, lg
        _check(lib().needle_run_batch_ids(self._h, _p(ids), _p(off), n, max_new, _p(mb), flags, _p(out), _p(lens)))
        return out, lens

    def debug_forward(self, enc_ids, dec_ids):
        """encode + teacher-forced decode steps -> (enc_out [T, d], logits [n_dec, V])."""
        e = np.ascontiguousarray(enc_ids, np.uint32)
        d = np.ascontiguousarray(dec_ids, np.uint32)
        enc = np.zeros((e.size, self.cfg["d_model"]), np.float32)
        lg = np.zeros((d.size, self.cfg["vocab_size"]), np.float32)
        _check(lib().needle_debug_forward(self._h, _p(e), e.size, _p(d) if d.size else None, d.size, _p(enc),
                                          _p(lg)))
        return enc, lg

    def prepare_batch(self, ids, offsets, max_new, mask_bits=None, flags=0):
        return Batch(self, ids, offsets, max_new, mask_bits, flags)


class Batch:
    """needle_batch_prepare / run / results (inputs uploaded once)."""

    def __init__(self, eng, ids, offsets, max_new, mask_bits=None, flags=0):
        self.eng = eng
        self._keep = (ids, offsets, mask_bits)
        ids_p = ids if isinstance(ids, int) else _p(np.ascontiguousarray(ids, np.uint32))
        off = np.ascontiguousarray(offsets, np.uint64)
        self._keep += (off,)
        mb = mask_bits if (mask_bits is None or isinstance(mask_bits, int)) else _p(mask_bits)
        self.n = off.size - 1
        self.max_new = max_new
        self._b = lib().needle_batch_prepare(eng._h, ids_p, _p(off), self.n, max_new, mb, flags)
        if not self._b:
            raise NeedleError(last_error() or "prepare failed")

    def run(self):
        _check(lib().needle_batch_run(self._b))

    def sync(self):
        _check(lib().needle_batch_sync(self._b))

    def begin(self):
        """Prefill; decode steps then run one at a time with step()."""
        _check(lib().needle_batch_begin(self._b))

    def set_step_mask(self, step, rows):
        r = np.ascontiguousarray(rows, np.uint64)
        _check(lib().needle_batch_set_step_mask(self._b, int(step), _p(r)))

    def step(self):
        """-> (tokens [n], lens [n], done [n]) of the decode step just run."""
        t = np.zeros(self.n, np.uint32)
        ln = np.zeros(self.n, np.uint32)
        d = np.zeros(self.n, np.uint8)
        _check(lib().needle_batch_step(self._b, _p(t), _p(ln), _p(d)))
        return t, ln, d

    def results(self):
        out = np.zeros((self.n, self.max_new), np.uint32)
        lens = np.zeros(self.n, np.uint32)
        _check(lib().needle_batch_results(self._b, _p(out), _p(lens)))
        return out, lens

    @property
    def stream(self):
        return lib().needle_batch_stream(self._b)

    def kernel_launches(self):
        return int(lib().needle_batch_kernel_launches(self._b))

    def time_kernel(self, kernel_class):
        """0 none, 1 cross-attention, 2 prefill matmul, 3 decode matmul, 4 head, 5 encoder attention,
        6 decoder self-attention, 7 elementwise kernels."""
        _check(lib().needle_batch_time_kernel(self._b, int(kernel_class)))

    def kernel_timing(self):
        """(ms_total, launches, flops, bytes) of the timed class over the last run."""
        ms, fl, by = C.c_double(), C.c_double(), C.c_double()
        n = C.c_int64()
        _check(lib().needle_batch_kernel_timing(self._b, C.byref(ms), C.byref(n), C.byref(fl), C.byref(by)))
        return ms.value, n.value, fl.value, by.value

    def close(self):
        if getattr(self, "_b", None):
            lib().needle_batch_free(self._b)
            self._b = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


(TIME_CROSS_ATTENTION, TIME_PREFILL_MATMUL, TIME_DECODE_MATMUL, TIME_HEAD, TIME_ENCODER_ATTENTION,
 TIME_SELF_ATTENTION, TIME_ELEMENTWISE) = 1, 2, 3, 4, 5, 6, 7


def shard_requests(offsets, shards):
    off = np.ascontiguousarray(offsets, np.uint64)
    out = np.zeros(off.size - 1, np.int32)
    _check(lib().needle_shard_requests(_p(off), off.size - 1, int(shards), _p(out)))
    return out


# ── kernel-level ops on device pointers (ints) ──
INT4_OVERLAP = 1


def int4_matmul(x_ptr, M, K, w_ptr, s_ptr, N, G, y_ptr, stream=None, overlap=False):
    """y[M][N] = x[M][K] @ W on device pointers (QuantizedWeight::matmul).
    overlap: launch with programmatic dependent launch (weights must not be
    written by work still in flight in the stream)."""
    if overlap:
        _check(lib().needle_int4_matmul_ex(x_ptr, M, K, w_ptr, s_ptr, N, G, y_ptr, INT4_OVERLAP, stream))
    else:
        _check(lib().needle_int4_matmul(x_ptr, M, K, w_ptr, s_ptr, N, G, y_ptr, stream))


class Int4Plan:
    """A prepared INT4 weight (device pointers in the reference layout) for
    repeated asynchronous matmuls of up to max_m rows."""

    def __init__(self, w_ptr, s_ptr, K, N, G, max_m, stream=None):
        self.K, self.N, self.max_m = K, N, max_m
        self._h = lib().needle_int4_plan_create(w_ptr, s_ptr, K, N, G, max_m, stream)
        if not self._h:
            raise NeedleError(last_error() or "needle_int4_plan_create failed")

    def matmul(self, x_ptr, M, y_ptr, stream=None, overlap=False):
        _check(lib().needle_int4_plan_matmul(self._h, x_ptr, M, y_ptr, INT4_OVERLAP if overlap else 0, stream))

    def status(self):
        _check(lib().needle_int4_plan_status(self._h))

    def close(self):
        if self._h:
            lib().needle_int4_plan_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def int4_quantize(w_ptr, K, N, data_ptr, scales_ptr, stream=None):
    _check(lib().needle_int4_quantize(w_ptr, K, N, data_ptr, scales_ptr, stream))


def int4_dequantize(data_ptr, scales_ptr, K, N, G, out_ptr, stream=None):
    _check(lib().needle_int4_dequantize(data_ptr, scales_ptr, K, N, G, out_ptr, stream))


def ffn_forward(x_ptr, T, d, ff, g, u, dn, act, out_ptr, stream=None):
    _check(lib().needle_ffn_forward(x_ptr, T, d, ff, g[0], g[1], u[0], u[1], dn[0], dn[1], act, out_ptr, stream))


class FfnPlan:
    """A prepared MLP block (needle_ffn_plan_*): gate / up / down as
    (packed, scales) device-pointer pairs in the reference layout; forward()
    is asynchronous and allocates nothing."""

    def __init__(self, d, ff, g, u, dn, max_t, stream=None):
        self.d, self.ff, self.max_t = d, ff, max_t
        self._h = lib().needle_ffn_plan_create(d, ff, g[0], g[1], u[0], u[1], dn[0], dn[1], max_t, stream)
        if not self._h:
            raise NeedleError(last_error() or "needle_ffn_plan_create failed")

    def forward(self, x_ptr, T, act, out_ptr, stream=None):
        _check(lib().needle_ffn_plan_forward(self._h, x_ptr, T, act, out_ptr, stream))

    def status(self):
        _check(lib().needle_ffn_plan_status(self._h))

    def close(self):
        if getattr(self, "_h", None):
            lib().needle_ffn_plan_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SafeTensors:
    """The library's SafeTensors reader (SafeTensors::from_bytes / get_metadata
    / get_f32 of crates/needle-infer/src/safetensors.rs) on a bytes buffer."""

    def __init__(self, data):
        self._buf = np.frombuffer(bytes(data), np.uint8)
        self._h = lib().needle_safetensors_parse(_p(self._buf) if self._buf.size else None, self._buf.size)
        if not self._h:
            raise NeedleError(last_error() or "SafeTensors parse failed")

    def get_metadata(self, key):
        v = lib().needle_safetensors_metadata(self._h, key.encode())
        return None if v is None else v.decode()

    def get_f32(self, name):
        n = lib().needle_safetensors_get_f32(self._h, name.encode(), None, 0)
        if n == C.c_size_t(-1).value:
            return None
        out = np.zeros(n, np.float32)
        lib().needle_safetensors_get_f32(self._h, name.encode(), _p(out), n)
        return out

    def close(self):
        if getattr(self, "_h", None):
            lib().needle_safetensors_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ffn_forward_noalloc(x_ptr, T, d, ff, g, u, dn, act, out_ptr, stream=None):
    """As ffn_forward, with the hidden activation in the library's fixed device
    array (no allocation; T * d_ff <= 1,048,576; overlapping calls race)."""
    _check(lib().needle_ffn_forward_noalloc(x_ptr, T, d, ff, g[0], g[1], u[0], u[1], dn[0], dn[1], act, out_ptr,
                                            stream))


# ── text front end (tokenizer, tool JSON, constrained decoding) ─────────────

def _take_str(r):
    if not r:
        raise NeedleError(last_error() or "needle call failed")
    s = C.string_at(r).decode()
    lib().needle_free_str(r)
    return s


class Vocab:
    """SentencePiece vocabulary (Vocabulary of tokenizer.rs)."""

    def __init__(self, text=None, _handle=None, _owner=None):
        self._own = _handle is None
        self._owner = _owner
        if _handle is None:
            b = text.encode() if isinstance(text, str) else bytes(text)
            _handle = lib().needle_vocab_parse(b, len(b))
            if not _handle:
                raise NeedleError(last_error() or "needle_vocab_parse failed")
        self._h = _handle

    def __len__(self):
        return lib().needle_vocab_size(self._h)

    def encode(self, text):
        b = text.encode()
        n = lib().needle_vocab_encode(self._h, b, None, 0)
        if n == C.c_size_t(-1).value:
            raise NeedleError("invalid text")
        out = np.zeros(max(n, 1), np.uint32)
        lib().needle_vocab_encode(self._h, b, _p(out), n)
        return out[:n].tolist()

    def decode(self, ids):
        a = np.ascontiguousarray(ids, np.uint32)
        return _take_str(lib().needle_vocab_decode(self._h, _p(a) if a.size else None, a.size))

    def close(self):
        if self._own and getattr(self, "_h", None):
            lib().needle_vocab_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def snake_case(name):
    return _take_str(lib().needle_snake_case(name.encode()))


def tools_encoder_text(tools_json):
    """The tools JSON as the encoder sees it (snake_case names, compact)."""
    return _take_str(lib().needle_tools_encoder_text(tools_json.encode()))


def restore_tool_names(tools_json, output):
    return _take_str(lib().needle_tools_restore_names(tools_json.encode(), output.encode()))


class Constraint:
    """ConstrainedDecoder of constrained.rs over a tools JSON."""

    FREE, IN_NAME, IN_ARG_KEY = 0, 1, 2

    def __init__(self, tools_json, vocab):
        self._vocab = vocab
        self._h = lib().needle_constraint_new(tools_json.encode(), vocab._h)
        if not self._h:
            raise NeedleError(last_error() or "needle_constraint_new failed")

    def update(self, token):
        _check(lib().needle_constraint_update(self._h, int(token)))

    def feed(self, data):
        b = data.encode() if isinstance(data, str) else bytes(data)
        _check(lib().needle_constraint_feed(self._h, b, len(b)))

    def mask(self, vocab_size):
        """-> (uint64 bitmap [ceil(V/64)], constrained?)"""
        bits = np.zeros((vocab_size + 63) // 64, np.uint64)
        rc = lib().needle_constraint_mask(self._h, vocab_size, _p(bits))
        if rc < 0:
            raise NeedleError("needle_constraint_mask failed")
        return bits, rc == 1

    @property
    def state(self):
        return lib().needle_constraint_state(self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().needle_constraint_free(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
