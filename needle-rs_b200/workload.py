"""Seeded synthetic workloads for the needle path (weights, prompts, masks).

The reference's real checkpoint and datasets are not available, so the
benchmark and the GPU parity tests use random-init models at the shipped
config dims (crates/needle-core/src/config.rs:46-69) in the reference's own
file format (tools/export.py:14-30, 160-246):
  projections  pre-quantized INT4 ("I4", shape [in_pad/2, out]) with codes
               uniform in [-8, 7] and f32 ".scale" [groups, out] uniform in
               [0.005, 0.02]
  embedding    N(0, 0.05^2) stored as BF16 (truncated, like export.to_bf16)
  norms        uniform in [-0.1, 0.1]; gates uniform in [-1, 1]
Everything is a pure function of the seed, so the GPU run and the CPU oracle
see identical inputs.
"""
import json
import struct

import numpy as np

DEFAULT_CFG = dict(d_model=512, num_heads=8, num_kv_heads=4, num_encoder_layers=12, num_decoder_layers=8,
                   vocab_size=8192, max_enc_len=1024, max_dec_len=512, ffn_dim=2048, no_feedforward=True,
                   activation="drelu", rope_theta=10000.0)


def write_safetensors(tensors, path=None, metadata=None):
    """tensors: {name: (dtype, shape, bytes)} -> SafeTensors bytes (and file if path)."""
    header = {}
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    off = 0
    parts = []
    for name, (dt, shape, data) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        parts.append(data)
        off += len(data)
    hj = json.dumps(header, separators=(",", ":")).encode()
    blob = struct.pack("<Q", len(hj)) + hj + b"".join(parts)
    if path:
        with open(path, "wb") as f:
            f.write(blob)
    return blob


def pack_codes(codes):
    """codes [K_pad, N] int in [-8, 7] -> reference layout bytes [K_pad/2, N]
    (low nibble = even row, high nibble = odd row; quant.rs:93-118)."""
    c = (np.asarray(codes).astype(np.int16) & 0xF).astype(np.uint8)
    return (c[0::2] | (c[1::2] << 4)).astype(np.uint8)


def random_int4(rng, K, N):
    """Random pre-quantized weight: (packed [K_pad/2, N] u8, scales [G, N] f32)."""
    gs = min(32, K)
    kp = K + (gs - K % gs) % gs
    codes = rng.integers(-8, 8, size=(kp, N), dtype=np.int8)
    scales = rng.uniform(0.005, 0.02, size=(kp // gs, N)).astype(np.float32)
    return pack_codes(codes), scales


def to_bf16_bytes(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()


def random_model(seed=0, path=None, contrastive=None, **overrides):
    """SafeTensors bytes of a random-init model (config overrides allowed).
    contrastive=(hidden_dim, contrastive_dim) adds the contrastive head's F32
    tensors (contrastive_hidden_kernel [d, h], contrastive_hidden_bias [h],
    contrastive_proj_kernel [h, c]), drawn after every other tensor."""
    cfg = dict(DEFAULT_CFG)
    cfg.update(overrides)
    rng = np.random.default_rng(seed)
    d, H, KVH = cfg["d_model"], cfg["num_heads"], cfg["num_kv_heads"]
    hd = d // H
    V, ff = cfg["vocab_size"], cfg["ffn_dim"]
    T = {}

    def f32(name, a):
        a = np.asarray(a, np.float32)
        T[name] = ("F32", list(a.shape), a.tobytes())

    def q(name, K, N):
        packed, scales = random_int4(rng, K, N)
        T[name] = ("I4", list(packed.shape), packed.tobytes())
        T[name + ".scale"] = ("F32", list(scales.shape), scales.tobytes())

    def attn(p):
        q(p + ".wq", d, H * hd)
        q(p + ".wk", d, KVH * hd)
        q(p + ".wv", d, KVH * hd)
        q(p + ".wo", H * hd, d)
        f32(p + ".q_norm", rng.uniform(-0.1, 0.1, hd))
        f32(p + ".k_norm", rng.uniform(-0.1, 0.1, hd))

    def ffn(p):
        f32(p + ".ffn_gate", [rng.uniform(-1, 1)])
        f32(p + ".ffn_norm", rng.uniform(-0.1, 0.1, d))
        q(p + ".ffn.gate_proj", d, ff)
        q(p + ".ffn.up_proj", d, ff)
        q(p + ".ffn.down_proj", ff, d)

    emb = (rng.standard_normal((V, d)) * 0.05).astype(np.float32)
    T["embedding"] = ("BF16", [V, d], to_bf16_bytes(emb))
    f32("encoder_final_norm", rng.uniform(-0.1, 0.1, d))
    f32("decoder_final_norm", rng.uniform(-0.1, 0.1, d))
    nf = str(cfg["no_feedforward"]) in ("True", "true", "1")
    for i in range(cfg["num_encoder_layers"]):
        p = f"encoder.{i}"
        f32(p + ".norm", rng.uniform(-0.1, 0.1, d))
        f32(p + ".self_attn_gate", [rng.uniform(-1, 1)])
        attn(p + ".self_attn")
        if not nf:
            ffn(p)
    for i in range(cfg["num_decoder_layers"]):
        p = f"decoder.{i}"
        f32(p + ".self_attn_norm", rng.uniform(-0.1, 0.1, d))
        f32(p + ".cross_attn_norm", rng.uniform(-0.1, 0.1, d))
        f32(p + ".self_attn_gate", [rng.uniform(-1, 1)])
        f32(p + ".cross_attn_gate", [rng.uniform(-1, 1)])
        attn(p + ".self_attn")
        attn(p + ".cross_attn")
        if not nf:
            ffn(p)
    if contrastive is not None:
        h, c = contrastive
        f32("contrastive_hidden_kernel", rng.standard_normal((d, h)) / np.sqrt(d))
        f32("contrastive_hidden_bias", rng.uniform(-0.1, 0.1, h))
        f32("contrastive_proj_kernel", rng.standard_normal((h, c)) / np.sqrt(h))
    return write_safetensors(T, path, metadata=cfg)


def random_prompts(n, lo, hi, vocab, seed):
    """n prompts with lengths uniform in [lo, hi] and ids uniform over vocab
    -> (ids uint32 concatenated, offsets uint64 [n+1])."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n)
    off = np.zeros(n + 1, np.uint64)
    np.cumsum(lens, out=off[1:])
    ids = rng.integers(0, vocab, size=int(off[-1]), dtype=np.uint32)
    return ids, off


def random_masks(n_req, max_new, vocab, frac=0.05, seed=0):
    """Per-(request, step) vocabulary bitmaps: each token allowed with
    probability `frac`, plus one forced token so at least one is always
    allowed.  -> uint64 [n_req, max_new, ceil(vocab/64)]."""
    rng = np.random.default_rng(seed)
    W = (vocab + 63) // 64
    out = np.zeros((n_req, max_new, W), np.uint64)
    thr = int(round(frac * 65536))
    chunk = max(1, (1 << 26) // max(1, max_new * vocab))
    for r0 in range(0, n_req, chunk):
        r1 = min(n_req, r0 + chunk)
        n = (r1 - r0) * max_new * vocab
        allowed = np.frombuffer(rng.bytes(2 * n), np.uint16).reshape(r1 - r0, max_new, vocab) < thr
        forced = rng.integers(0, vocab, size=(r1 - r0, max_new))
        np.put_along_axis(allowed, forced[..., None], True, axis=2)
        padded = np.zeros((r1 - r0, max_new, W * 64), bool)
        padded[..., :vocab] = allowed
        out[r0:r1] = np.packbits(padded, axis=2, bitorder="little").view(np.uint64)
    return out


def int4_case(M, N, K, seed=0):
    """The INT4 matmul workload (activations N(0,1) [M, K]; codes U{-8..7};
    scales U(0.005, 0.02) per group of 32 along K) -> (x, packed, scales)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    packed, scales = random_int4(rng, K, N)
    return x, packed, scales


SPECIAL_PIECES = ["<pad>", "</s>", "<s>", "<unk>", "<tool_call>", "<tools>"]


def random_vocab(size=8192, seed=0):
    """A SentencePiece-style vocabulary text ("piece\\tscore" per line) of
    `size` pieces, in the layout of the shipped vocab: the six special tokens
    (ids 0-5), the 256 byte-fallback pieces <0xXX>, the base characters
    (U+2581, printable ASCII, a few non-ASCII letters), then merged pieces
    drawn from words and JSON fragments with scores -(merge rank)."""
    rng = np.random.default_rng(seed)
    pieces = list(SPECIAL_PIECES) + ["<0x%02X>" % b for b in range(256)]
    base = ["\u2581"] + [chr(c) for c in range(0x21, 0x7F)] + list("éàüßñ")
    pieces += base
    scores = [0.0] * len(pieces)
    words = ["name", "arguments", "get", "weather", "location", "unit", "city", "search", "query", "time",
             "set", "alarm", "send", "message", "email", "book", "flight", "from", "to", "date", "the", "what",
             "is", "of", "for", "and", "please", "new", "york", "paris", "celsius", "call", "tool", "value"]
    letters = "abcdefghijklmnopqrstuvwxyz"
    for _ in range(600):
        words.append("".join(rng.choice(list(letters), int(rng.integers(2, 9)))))
    frags = ['{"', '":"', '","', '":{', '"}', '}}', '}]', '[{"', '":', ',"', '":"get', '_', '":[']
    cand = []
    seen = set(pieces)
    for w in words:
        for form in (w, "\u2581" + w, w.capitalize(), "\u2581" + w.capitalize(), "_" + w):
            for L in range(2, min(len(form), 9) + 1):
                for i in range(0, len(form) - L + 1):
                    cand.append(form[i:i + L])
    cand += frags
    rng.shuffle(cand)
    # shorter pieces first so that longer ones are reachable through merges
    cand.sort(key=len)
    rank = 1
    for c in cand:
        if len(pieces) >= size:
            break
        if c in seen:
            continue
        seen.add(c)
        pieces.append(c)
        scores.append(-float(rank))
        rank += 1
    while len(pieces) < size:  # pad with unused pieces
        pieces.append("<extra_%d>" % len(pieces))
        scores.append(-float(rank))
        rank += 1
    return "".join("%s\t%s\n" % (p, repr(sc) if sc != int(sc) else "%d" % int(sc)) for p, sc in zip(pieces, scores))
