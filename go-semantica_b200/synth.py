"""Seeded synthetic inputs with the shapes of the reference's workloads.

The EmbeddingGemma-300M weights are not available on this machine (the
reference ships a Git-LFS pointer in place of model/embeddinggemma-300m-Q8_0.gguf),
so every model used by the tests and the bench is a synthetic GGUF v3 file with
the same architecture metadata and tensor names the reference loader reads
(internal/runtime/model.go:424-517, internal/runtime/model_int8.go:54-119,
internal/gguf/reader.go:98-178):

* Q8_0 tensors: per 32-element block an fp16 scale d and 32 int8 codes; codes
  uniform in [-127, 127], d = fp16(max|N(0, 0.02)| over the block's 32 draws / 127).
* Norm weights: F32, 1 + N(0, 0.1) (the reference multiplies by w, not 1+w,
  internal/kernels/norm.go:34).
* A small vocabulary of token strings; ids 0-3 are the special tokens
  (pad/eos/bos/unk; bos = 2, eos = 1 as in testdata/reference_token_ids.json),
  "non-special" ids are >= 4.

Corpus and query vectors for search/brute are seeded N(0, 1) draws.
"""
from __future__ import annotations

import os
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3
DTYPE_F32 = 0
DTYPE_Q8_0 = 8
ALIGN = 32

BOS_ID = 2
EOS_ID = 1
FIRST_NON_SPECIAL = 4

# EmbeddingGemma-300M shapes (the config parseConfig reads, internal/runtime/
# model.go:424-517): hidden 768, 24 blocks, 3 query heads, 1 KV head,
# head_dim 256, FFN 1152, context 2048, vocabulary 262144.
GEMMA_300M = dict(embed_dim=768, num_layers=24, num_heads=3, num_kv_heads=1, interm_dim=1152,
                  context_length=2048, vocab_size=262144, norm_eps=1e-6, rope_base=10000.0)


def _kv_string(key: str, val: str) -> bytes:
    kb, vb = key.encode(), val.encode()
    return struct.pack("<Q", len(kb)) + kb + struct.pack("<I", 8) + struct.pack("<Q", len(vb)) + vb


def _kv_u32(key: str, val: int) -> bytes:
    kb = key.encode()
    return struct.pack("<Q", len(kb)) + kb + struct.pack("<II", 4, val)


def _kv_f32(key: str, val: float) -> bytes:
    kb = key.encode()
    return struct.pack("<Q", len(kb)) + kb + struct.pack("<If", 6, val)


def _kv_str_array(key: str, vals) -> bytes:
    kb = key.encode()
    parts = [struct.pack("<Q", len(kb)), kb, struct.pack("<IIQ", 9, 8, len(vals))]
    for v in vals:
        vb = v.encode()
        parts.append(struct.pack("<Q", len(vb)))
        parts.append(vb)
    return b"".join(parts)


def q8_0_blocks(rng: np.random.Generator, rows: int, cols: int, chunk_rows: int = 4096) -> np.ndarray:
    """Random Q8_0 tensor of `rows` output rows x `cols` inputs, as raw bytes
    [rows, cols/32, 34] (fp16 scale little-endian, then 32 int8 codes)."""
    assert cols % 32 == 0
    nb = cols // 32
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        n = r1 - r0
        qs = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int16).astype(np.int8)
        draws = np.abs(rng.standard_normal(size=(n, nb, 32), dtype=np.float32)) * np.float32(0.02)
        d = (draws.max(axis=2) / np.float32(127.0)).astype(np.float16)
        out[r0:r1, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
        out[r0:r1, :, 2:] = qs.view(np.uint8)
    return out


def write_gguf(path: str, seed: int = 1234, vocab_size: int | None = None, num_layers: int | None = None,
               dense_head: bool = False, **overrides) -> str:
    """Writes a synthetic EmbeddingGemma-shaped GGUF v3 file and returns its path.

    dense_head adds the EmbeddingGemma dense head the reference does not read
    (dense_2.weight: embed -> 4 embed, dense_3.weight: 4 embed -> embed, Q8_0,
    drawn after every other tensor so the rest of the file is unchanged) and
    the sliding-window metadata key (512 tokens), for the model-faithful mode."""
    cfg = dict(GEMMA_300M)
    if vocab_size is not None:
        cfg["vocab_size"] = vocab_size
    if num_layers is not None:
        cfg["num_layers"] = num_layers
    cfg.update(overrides)
    H, F, L = cfg["embed_dim"], cfg["interm_dim"], cfg["num_layers"]
    nh, nkv = cfg["num_heads"], cfg["num_kv_heads"]
    hd = H // nh
    V = cfg["vocab_size"]
    rng = np.random.default_rng(seed)
    arch = "gemma-embedding"

    tensors = []  # (name, dtype, dims[ne0, ne1...], bytes)

    def add_q8(name, k_in, n_out):
        tensors.append((name, DTYPE_Q8_0, [k_in, n_out], q8_0_blocks(rng, n_out, k_in)))

    def add_norm(name, n):
        w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        tensors.append((name, DTYPE_F32, [n], w))

    add_q8("token_embd.weight", H, V)
    add_norm("output_norm.weight", H)
    for l in range(L):
        p = f"blk.{l}."
        add_norm(p + "attn_norm.weight", H)
        add_q8(p + "attn_q.weight", H, nh * hd)
        add_q8(p + "attn_k.weight", H, nkv * hd)
        add_q8(p + "attn_v.weight", H, nkv * hd)
        add_q8(p + "attn_output.weight", H, H)
        add_norm(p + "attn_q_norm.weight", hd)
        add_norm(p + "attn_k_norm.weight", hd)
        add_norm(p + "post_attention_norm.weight", H)
        add_norm(p + "ffn_norm.weight", H)
        add_q8(p + "ffn_gate.weight", H, F)
        add_q8(p + "ffn_up.weight", H, F)
        add_q8(p + "ffn_down.weight", F, H)
        add_norm(p + "post_ffw_norm.weight", H)
    if dense_head:
        add_q8("dense_2.weight", H, 4 * H)
        add_q8("dense_3.weight", 4 * H, H)

    tokens = ["<pad>", "<eos>", "<bos>", "<unk>"] + [f"t{i}" for i in range(4, V)]
    kv = [
        _kv_string("general.architecture", arch),
        _kv_u32(f"{arch}.embedding_length", H),
        _kv_u32(f"{arch}.block_count", L),
        _kv_u32(f"{arch}.attention.head_count", nh),
        _kv_u32(f"{arch}.attention.head_count_kv", nkv),
        _kv_u32(f"{arch}.feed_forward_length", F),
        _kv_u32(f"{arch}.context_length", cfg["context_length"]),
        _kv_f32(f"{arch}.attention.layer_norm_rms_epsilon", cfg["norm_eps"]),
        _kv_f32(f"{arch}.rope.freq_base", cfg["rope_base"]),
        _kv_str_array("tokenizer.ggml.tokens", tokens),
    ]
    if dense_head:
        kv.append(_kv_u32(f"{arch}.attention.sliding_window", 512))
    infos = []
    offset = 0
    for name, dt, dims, arr in tensors:
        nb = name.encode()
        infos.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
                     + b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", dt, offset))
        offset += arr.nbytes
        offset = (offset + ALIGN - 1) // ALIGN * ALIGN
    header = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(kv))
    meta = header + b"".join(kv) + b"".join(infos)
    pad = (-len(meta)) % ALIGN
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(meta)
        f.write(b"\0" * pad)
        pos = 0
        for _, _, _, arr in tensors:
            b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
            f.write(b.tobytes())
            pos += b.nbytes
            p2 = (-pos) % ALIGN
            f.write(b"\0" * p2)
            pos += p2
    os.replace(tmp, path)
    return path


def cached_gguf(directory: str, seed: int = 1234, vocab_size: int | None = None,
                num_layers: int | None = None, dense_head: bool = False) -> str:
    """Path of a synthetic model in `directory`, written on first use."""
    v = vocab_size or GEMMA_300M["vocab_size"]
    l = num_layers or GEMMA_300M["num_layers"]
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"synth-gemma-s{seed}-v{v}-l{l}{'-dense' if dense_head else ''}.gguf")
    if not os.path.exists(path):
        write_gguf(path, seed=seed, vocab_size=v, num_layers=l, dense_head=dense_head)
    return path


def token_batch(seed: int, lengths, vocab_size: int) -> tuple[np.ndarray, np.ndarray]:
    """Packed token ids (BOS then uniform non-special ids) and offsets [B+1]."""
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, dtype=np.int64)
    offsets = np.zeros(len(lengths) + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(lengths)
    ids = rng.integers(FIRST_NON_SPECIAL, vocab_size, size=int(offsets[-1]), dtype=np.int64).astype(np.int32)
    ids[offsets[:-1]] = BOS_ID
    return ids, offsets


def ragged_lengths(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Sequence lengths uniform in [lo, hi]."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


def normal_vectors(seed: int, n: int, dim: int, chunk: int = 1 << 18) -> np.ndarray:
    """n x dim float32 N(0,1) draws."""
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), dtype=np.float32)
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        out[r0:r1] = rng.standard_normal(size=(r1 - r0, dim), dtype=np.float32)
    return out
