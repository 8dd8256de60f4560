"""Synthetic .ember models with the shapes of the benchmark configurations.

There are no checkpoints offline, so every model the tests and the benchmark use
is written here: weights N(0, 0.02) as float32 from ``numpy.random.default_rng``
(norm weights 1.0, attention biases N(0, 0.01)), quantized to Q8_0 / Q4_0 with
this library's host quantizers (byte-identical to emberllm's ``ember quantize``;
tests/test_quant_file.py checks that), and laid out in emberllm's file format
(ref src/ember.h:1-14, tools/convert.py:57-112): 256-byte header, tokenizer blob,
8-aligned tensor table, 64-aligned tensor data.

The tokenizer blob is a minimal SentencePiece table (ref src/tokenizer.c:124-140:
int32 max_len, then per token float32 score, int32 length, bytes), so emberllm's
CLI can open the files too.
"""
import ctypes
import hashlib
import json
import os
import struct

import numpy as np

DT_F32, DT_Q8_0, DT_Q4_0 = 0, 1, 2
FLAG_TIED, FLAG_QK_NORM = 1, 2
ROPE_INTERLEAVED, ROPE_NEOX = 0, 1

# the four BASELINE architectures (dims from the benchmark configurations) and
# small variants of each for tests
CONFIGS = {
    "stories110m": dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, n_kv_heads=12,
                        head_dim=64, vocab_size=32000, max_seq_len=1024, rope_theta=10000.0,
                        norm_eps=1e-5, rope_style=ROPE_INTERLEAVED, tied=True, qk_norm=False,
                        bias=False, quant="q8_0"),
    "smollm2-135m": dict(dim=576, hidden_dim=1536, n_layers=30, n_heads=9, n_kv_heads=3,
                         head_dim=64, vocab_size=49152, max_seq_len=8192, rope_theta=100000.0,
                         norm_eps=1e-5, rope_style=ROPE_NEOX, tied=True, qk_norm=False,
                         bias=False, quant="q4_0"),
    "qwen2.5-0.5b": dict(dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2,
                         head_dim=64, vocab_size=151936, max_seq_len=32768, rope_theta=1e6,
                         norm_eps=1e-6, rope_style=ROPE_NEOX, tied=True, qk_norm=False,
                         bias=True, quant="q8_0"),
    "qwen3-0.6b": dict(dim=1024, hidden_dim=3072, n_layers=28, n_heads=16, n_kv_heads=8,
                       head_dim=128, vocab_size=151936, max_seq_len=40960, rope_theta=1e6,
                       norm_eps=1e-6, rope_style=ROPE_NEOX, tied=True, qk_norm=True,
                       bias=False, quant="q8_0"),
    # small cases: every code path at sizes the CPU oracle finishes in moments
    "tiny-llama": dict(dim=128, hidden_dim=320, n_layers=2, n_heads=4, n_kv_heads=4, head_dim=32,
                       vocab_size=512, max_seq_len=256, rope_theta=10000.0, norm_eps=1e-5,
                       rope_style=ROPE_INTERLEAVED, tied=False, qk_norm=False, bias=False,
                       quant="q8_0"),
    "tiny-qwen3": dict(dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64,
                       vocab_size=640, max_seq_len=512, rope_theta=1e6, norm_eps=1e-6,
                       rope_style=ROPE_NEOX, tied=True, qk_norm=True, bias=False, quant="q8_0"),
    "tiny-qwen2": dict(dim=96, hidden_dim=224, n_layers=2, n_heads=3, n_kv_heads=1, head_dim=32,
                       vocab_size=384, max_seq_len=256, rope_theta=1e6, norm_eps=1e-6,
                       rope_style=ROPE_NEOX, tied=True, qk_norm=False, bias=True, quant="q8_0"),
    "tiny-smol-q4": dict(dim=96, hidden_dim=256, n_layers=3, n_heads=3, n_kv_heads=1, head_dim=32,
                         vocab_size=320, max_seq_len=256, rope_theta=100000.0, norm_eps=1e-5,
                         rope_style=ROPE_NEOX, tied=True, qk_norm=False, bias=False,
                         quant="q4_0"),
    # eight query heads per kv head: the single-kernel decode attention path
    "tiny-mqa": dict(dim=256, hidden_dim=384, n_layers=2, n_heads=8, n_kv_heads=1, head_dim=32,
                     vocab_size=448, max_seq_len=256, rope_theta=10000.0, norm_eps=1e-5,
                     rope_style=ROPE_NEOX, tied=True, qk_norm=True, bias=False, quant="q8_0"),
    # long contexts: batched prefill in several chunks and softmax sums past 2048 terms
    "tiny-long": dict(dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64,
                      vocab_size=512, max_seq_len=4096, rope_theta=1e6, norm_eps=1e-6,
                      rope_style=ROPE_NEOX, tied=True, qk_norm=True, bias=False, quant="q8_0"),
    "tiny-f32": dict(dim=64, hidden_dim=160, n_layers=2, n_heads=2, n_kv_heads=2, head_dim=32,
                     vocab_size=256, max_seq_len=128, rope_theta=10000.0, norm_eps=1e-5,
                     rope_style=ROPE_INTERLEAVED, tied=False, qk_norm=False, bias=False,
                     quant="f32"),
}

_HEADER = struct.Struct("<4sIQ8iffIi4i2i2f4Q128s")
_ENTRY = struct.Struct("<48sii4iQQ")
assert _HEADER.size == 256 and _ENTRY.size == 88


def _pad(n, a):
    return (n + a - 1) // a * a


def tokenizer_blob(vocab):
    """A SentencePiece table emberllm's tokenizer can parse: <unk>, <s>, </s>,
    the 256 byte tokens, then placeholder pieces."""
    pieces = []
    for i in range(vocab):
        if i < 3:
            s = ["<unk>", "<s>", "</s>"][i]
        elif i < 259:
            s = "<0x%02X>" % (i - 3)
        else:
            s = "tok%d" % i
        pieces.append(s.encode())
    out = [struct.pack("<i", max(len(p) for p in pieces))]
    for i, p in enumerate(pieces):
        out.append(struct.pack("<fi", -float(i), len(p)))
        out.append(p)
    return b"".join(out)


def _tensor_specs(cfg):
    """(name, shape, kind) in file order; kind is 'w' (matrix), 'norm' or 'bias'."""
    d, h, hd = cfg["dim"], cfg["hidden_dim"], cfg["head_dim"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    specs = [("tok_embeddings", (cfg["vocab_size"], d), "w")]
    for l in range(cfg["n_layers"]):
        p = "layers.%d." % l
        specs += [(p + "attn_norm", (d,), "norm"), (p + "wq", (qd, d), "w"),
                  (p + "wk", (kvd, d), "w"), (p + "wv", (kvd, d), "w")]
        if cfg["bias"]:
            specs += [(p + "wq_bias", (qd,), "bias"), (p + "wk_bias", (kvd,), "bias"),
                      (p + "wv_bias", (kvd,), "bias")]
        if cfg["qk_norm"]:
            specs += [(p + "q_norm", (hd,), "norm"), (p + "k_norm", (hd,), "norm")]
        specs += [(p + "wo", (d, qd), "w"), (p + "ffn_norm", (d,), "norm"),
                  (p + "w1", (h, d), "w"), (p + "w2", (d, h), "w"), (p + "w3", (h, d), "w")]
    specs.append(("final_norm", (d,), "norm"))
    if not cfg["tied"]:
        specs.append(("lm_head", (cfg["vocab_size"], d), "w"))
    return specs


def _quantize(values, kind, lib):
    """fp32 rows -> Q8_0 / Q4_0 bytes through the library's host quantizers."""
    rows, cols = values.shape
    nb = cols // 32
    blk = 34 if kind == DT_Q8_0 else 18
    out = np.empty(rows * nb * blk, dtype=np.uint8)
    fn = lib.ember_quantize_q8_0 if kind == DT_Q8_0 else lib.ember_quantize_q4_0
    src = np.ascontiguousarray(values, dtype=np.float32)
    step = max(1, (1 << 22) // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        fn(src[r0:r1].ctypes.data, out[r0 * nb * blk:].ctypes.data, (r1 - r0) * cols)
    return out.tobytes()


def write_model(path, cfg, seed=0, quant=None, lib=None):
    """Write a synthetic model for ``cfg``; ``quant`` in {"f32", "q8_0", "q4_0"}
    (default: the config's). Returns the path."""
    quant = quant or cfg["quant"]
    if quant != "f32" and lib is None:
        from . import _lib
        lib = _lib.load()
    rng = np.random.default_rng(seed)
    tensors = []
    for name, shape, kind in _tensor_specs(cfg):
        if kind == "norm":
            vals = np.ones(shape, dtype=np.float32)
        else:
            scale = np.float32(0.02 if kind == "w" else 0.01)
            vals = rng.standard_normal(shape, dtype=np.float32) * scale
        dtype = DT_F32
        if kind == "w" and quant != "f32" and shape[1] % 32 == 0:
            dtype = DT_Q8_0
            if quant == "q4_0" and name not in ("tok_embeddings", "lm_head"):
                dtype = DT_Q4_0
        data = vals.astype("<f4").tobytes() if dtype == DT_F32 else _quantize(vals, dtype, lib)
        tensors.append((name, dtype, shape, data))

    blob = tokenizer_blob(cfg["vocab_size"])
    tok_off = 256
    table_off = _pad(tok_off + len(blob), 8)
    table_size = len(tensors) * 88
    data_off = _pad(table_off + table_size, 64)
    offsets, cur = [], data_off
    for t in tensors:
        cur = _pad(cur, 64)
        offsets.append(cur)
        cur += len(t[3])
    flags = (FLAG_TIED if cfg["tied"] else 0) | (FLAG_QK_NORM if cfg["qk_norm"] else 0)
    header = _HEADER.pack(
        b"EMBR", 1, data_off,
        cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
        cfg["head_dim"], cfg["vocab_size"], cfg["max_seq_len"],
        cfg["rope_theta"], cfg["norm_eps"], flags, cfg["rope_style"],
        1, 2, -1, len(tensors), 0, 40, 1.0, 0.9,
        tok_off, len(blob), table_off, table_size, b"\0" * 128)
    table = b"".join(
        _ENTRY.pack(name.encode(), dtype, len(shape), *(list(shape) + [1] * (4 - len(shape))),
                    offsets[i], len(data))
        for i, (name, dtype, shape, data) in enumerate(tensors))
    tmp = path + ".tmp%d" % os.getpid()
    with open(tmp, "wb") as f:
        f.write(header)
        f.write(blob)
        f.write(b"\0" * (table_off - f.tell()))
        f.write(table)
        f.write(b"\0" * (data_off - f.tell()))
        for i, (_, _, _, data) in enumerate(tensors):
            f.write(b"\0" * (offsets[i] - f.tell()))
            f.write(data)
    os.replace(tmp, path)
    return path


def cache_dir():
    d = os.environ.get("EMBER_CACHE_DIR") or os.path.join(
        os.path.expanduser("~"), ".cache", "ember_b200")
    os.makedirs(os.path.join(d, "models"), exist_ok=True)
    return os.path.join(d, "models")


def ensure_model(name, seed=0, quant=None, directory=None):
    """Path of the synthetic model ``name`` (generated once, then cached)."""
    cfg = CONFIGS[name]
    quant = quant or cfg["quant"]
    key = hashlib.sha256(json.dumps([cfg, seed, quant, 1], sort_keys=True).encode()).hexdigest()[:12]
    path = os.path.join(directory or cache_dir(), "%s-%s-s%d-%s.ember" % (name, quant, seed, key))
    if not os.path.exists(path):
        write_model(path, cfg, seed=seed, quant=quant)
    return path


def weight_bytes_per_token(cfg, quant=None):
    """Algorithmic weight bytes one decode step streams: every quantized matrix
    once (34/32 B per Q8_0 weight, 18/32 per Q4_0, 4 per fp32), lm_head (the
    embedding when tied), the fp32 norm and bias vectors, one embedding row."""
    quant = quant or cfg["quant"]
    total = 0
    per = {DT_F32: 4.0, DT_Q8_0: 34 / 32, DT_Q4_0: 18 / 32}
    emb_dt = DT_F32 if quant == "f32" else DT_Q8_0
    for name, shape, kind in _tensor_specs(cfg):
        n = int(np.prod(shape))
        if kind != "w":
            total += 4 * n
            continue
        dt = DT_F32
        if quant != "f32" and shape[1] % 32 == 0:
            dt = DT_Q8_0 if (quant == "q8_0" or name in ("tok_embeddings", "lm_head")) else DT_Q4_0
        if name == "tok_embeddings":
            total += per[dt] * shape[1]                 # one row gathered
            if cfg["tied"]:
                total += per[dt] * n                    # read again as lm_head
            continue
        total += per[dt] * n
    return int(total)
