"""ctypes binding of the CPU oracle (oracle/_build/libneedle_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py for the timed CPU baseline arm.  The product
(libneedle_c.so and its Python binding) never imports this module.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libneedle_oracle.so")

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, S, F, I = C.c_void_p, C.c_size_t, C.c_float, C.c_int
        sig = {
            "orc_quant_sizes": (None, [S, S, C.POINTER(S), C.POINTER(S)]),
            "orc_quantize": (None, [P, S, S, P, P]),
            "orc_dequantize": (None, [P, P, S, S, S, P]),
            "orc_matvec": (None, [P, P, S, S, S, P, P, I]),
            "orc_matmul": (None, [P, P, S, S, S, P, S, P, I]),
            "orc_sign_extend4": (I, [C.c_uint8]),
            "orc_zc_rms_norm": (None, [P, P, S]),
            "orc_rope_table": (None, [S, S, F, P, P]),
            "orc_rope_apply": (None, [P, P, S, P, S, S, S, S]),
            "orc_softmax": (None, [P, S]),
            "orc_sigmoid": (F, [F]),
            "orc_gelu": (F, [F]),
            "orc_ffn_forward": (None, [P, P, P, P, P, P, S, S, P, P, I]),
            "orc_model_load_file": (P, [C.c_char_p, C.c_char_p, S]),
            "orc_model_load_bytes": (P, [P, S, C.c_char_p, S]),
            "orc_model_free": (None, [P]),
            "orc_model_config": (None, [P, P]),
            "orc_forward": (I, [P, P, S, P, S, P, P]),
            "orc_generate": (S, [P, P, S, S, P, I, P, P, P]),
            "orc_run_batch": (I, [P, P, P, S, S, P, I, P, P, P, I, P]),
            "orc_kv_cache_push_count": (S, [S, S]),
            "orc_encode_contrastive": (S, [P, P, S, P]),
            "orc_contrastive_dim": (S, [P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def quant_sizes(in_feat, out_feat):
    db, ng = C.c_size_t(), C.c_size_t()
    lib().orc_quant_sizes(in_feat, out_feat, C.byref(db), C.byref(ng))
    return db.value, ng.value


def quantize(w):
    """quant.rs:63-128 on w [in_feat, out_feat] f32 -> (packed u8, scales [G, out] f32)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    in_f, out_f = w.shape
    db, ng = quant_sizes(in_f, out_f)
    data = np.zeros(db, np.uint8)
    scales = np.zeros((ng, out_f), np.float32)
    lib().orc_quantize(_p(w), in_f, out_f, _p(data), _p(scales))
    return data, scales


def dequantize(data, scales, in_feat, out_feat):
    out = np.zeros((in_feat, out_feat), np.float32)
    data = np.ascontiguousarray(data, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    lib().orc_dequantize(_p(data), _p(scales), in_feat, out_feat, scales.size // out_feat, _p(out))
    return out


def matmul(data, scales, in_feat, out_feat, x, path=1):
    """quant.rs:400-410 (path 1 = AVX2 order, 0 = scalar order); x [M, in_feat]."""
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    data = np.ascontiguousarray(data, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    y = np.zeros((x.shape[0], out_feat), np.float32)
    lib().orc_matmul(_p(data), _p(scales), in_feat, out_feat, scales.size // out_feat, _p(x), x.shape[0], _p(y), path)
    return y


def zc_rms_norm(x, scale):
    x = np.array(x, np.float32)
    s = np.ascontiguousarray(scale, np.float32)
    lib().orc_zc_rms_norm(_p(x), _p(s), x.size)
    return x


def rope_table(max_len, head_dim, base=10000.0):
    c = np.zeros((max_len, head_dim // 2), np.float32)
    s = np.zeros((max_len, head_dim // 2), np.float32)
    lib().orc_rope_table(max_len, head_dim, base, _p(c), _p(s))
    return c, s


def rope_apply(x, seq_len, num_heads, head_dim, offset, max_len=8, base=10000.0):
    c, s = rope_table(max(max_len, seq_len + offset), head_dim, base)
    x = np.array(x, np.float32)
    lib().orc_rope_apply(_p(c), _p(s), head_dim // 2, _p(x), seq_len, num_heads, head_dim, offset)
    return x


def softmax(x):
    x = np.array(x, np.float32)
    lib().orc_softmax(_p(x), x.size)
    return x


def ffn_forward(g, u, d, d_model, d_ff, x, act=0):
    """ffn.rs:19-56 for one token; g/u/d are (packed, scales) pairs."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(d_model, np.float32)
    lib().orc_ffn_forward(_p(g[0]), _p(g[1]), _p(u[0]), _p(u[1]), _p(d[0]), _p(d[1]),
                          d_model, d_ff, _p(x), _p(out), act)
    return out


class Model:
    """Oracle model loaded from a SafeTensors file or buffer."""

    def __init__(self, path=None, data=None):
        err = C.create_string_buffer(512)
        if path is not None:
            self.h = lib().orc_model_load_file(path.encode(), err, 512)
        else:
            buf = np.frombuffer(data, np.uint8)
            self.h = lib().orc_model_load_bytes(_p(buf), buf.size, err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        cfg = np.zeros(12, np.int64)
        lib().orc_model_config(self.h, _p(cfg))
        keys = ["d_model", "num_heads", "num_kv_heads", "num_layers", "num_dec_layers", "vocab_size",
                "max_enc_len", "max_dec_len", "ffn_dim", "no_feedforward", "activation", "head_dim"]
        self.cfg = dict(zip(keys, (int(v) for v in cfg)))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def forward(self, enc_ids, dec_ids):
        """encode + teacher-forced decode steps -> (enc_out [T, d], logits [n_dec, V])."""
        e = np.ascontiguousarray(enc_ids, np.uint32)
        dd = np.ascontiguousarray(dec_ids, np.uint32)
        enc = np.zeros((e.size, self.cfg["d_model"]), np.float32)
        lg = np.zeros((dd.size, self.cfg["vocab_size"]), np.float32)
        rc = lib().orc_forward(self.h, _p(e), e.size, _p(dd), dd.size, _p(enc), _p(lg))
        if rc != 0:
            raise ValueError("invalid token ids")
        return enc, lg

    @property
    def contrastive_dim(self):
        return lib().orc_contrastive_dim(self.h)

    def encode_contrastive(self, ids):
        """encode_contrastive (engine.rs:153-181) on token ids, or None
        without a contrastive head."""
        c = self.contrastive_dim
        if not c:
            return None
        e = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(c, np.float32)
        if lib().orc_encode_contrastive(self.h, _p(e) if e.size else None, e.size, _p(out)) != c:
            raise ValueError("invalid token ids")
        return out

    def generate(self, enc_ids, max_new, mask_bits=None, stop_on_eos=False, want_logits=False):
        e = np.ascontiguousarray(enc_ids, np.uint32)
        out = np.zeros(max_new, np.uint32)
        marg = np.zeros(max_new, np.float32)
        lg = np.zeros((max_new, self.cfg["vocab_size"]), np.float32) if want_logits else None
        mb = None if mask_bits is None else np.ascontiguousarray(mask_bits, np.uint64)
        n = lib().orc_generate(self.h, _p(e), e.size, max_new, _p(mb), int(stop_on_eos), _p(out), _p(marg), _p(lg))
        res = (out[:n], marg[:n])
        return res + (lg[:n],) if want_logits else res

    def run_batch(self, ids, offsets, max_new, mask_bits=None, stop_on_eos=False, n_threads=1, want_tops=False):
        """-> (ids [n, max_new], lens [n], top-2 margins [n, max_new][, top
        masked logit of each step [n, max_new] when want_tops])."""
        ids = np.ascontiguousarray(ids, np.uint32)
        offsets = np.ascontiguousarray(offsets, np.uint64)
        n_req = offsets.size - 1
        out = np.zeros((n_req, max_new), np.uint32)
        lens = np.zeros(n_req, np.uint32)
        marg = np.zeros((n_req, max_new), np.float32)
        tops = np.zeros((n_req, max_new), np.float32) if want_tops else None
        mb = None if mask_bits is None else np.ascontiguousarray(mask_bits, np.uint64)
        rc = lib().orc_run_batch(self.h, _p(ids), _p(offsets), n_req, max_new, _p(mb), int(stop_on_eos),
                                 _p(out), _p(lens), _p(marg), n_threads, _p(tops))
        if rc != 0:
            raise ValueError("invalid request")
        return (out, lens, marg, tops) if want_tops else (out, lens, marg)
