"""Deterministic synthetic Hugging Face checkpoints (safetensors) for the
converter tests: every tensor name and shape of Qwen2.5-0.5B (BF16) and
GPT-2 124M (F32), values from a counter-based splitmix64 stream per tensor
(seed, tensor index), so the bytes depend on nothing but the seed.

Values are uniform in [-0.05, 0.05): small enough that part of them fall
into FP16's subnormal range, which the FP16 rounding must keep.  Tensors
are stored in a shuffled order, not the converters' write order, so the
converters must follow the header's data_offsets.
"""
import json
import struct
from concurrent.futures import ThreadPoolExecutor

import numpy as np

M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
GOLD = np.uint64(0x9E3779B97F4A7C15)
BLOCK = 1 << 22


def qwen_tensors():
    V, C, NL, KVD, FC = 151936, 896, 24, 128, 4864
    t = [("model.embed_tokens.weight", [V, C]), ("model.norm.weight", [C])]
    for i in range(NL):
        p = f"model.layers.{i}."
        t += [(p + "input_layernorm.weight", [C]), (p + "self_attn.q_proj.weight", [C, C]),
              (p + "self_attn.q_proj.bias", [C]), (p + "self_attn.k_proj.weight", [KVD, C]),
              (p + "self_attn.k_proj.bias", [KVD]), (p + "self_attn.v_proj.weight", [KVD, C]),
              (p + "self_attn.v_proj.bias", [KVD]), (p + "self_attn.o_proj.weight", [C, C]),
              (p + "post_attention_layernorm.weight", [C]), (p + "mlp.gate_proj.weight", [FC, C]),
              (p + "mlp.up_proj.weight", [FC, C]), (p + "mlp.down_proj.weight", [C, FC])]
    return t


def gpt2_tensors():
    V, C, NL, FC = 50257, 768, 12, 3072
    t = [("wte.weight", [V, C]), ("wpe.weight", [1024, C]), ("ln_f.weight", [C]), ("ln_f.bias", [C])]
    for i in range(NL):
        h = f"h.{i}."
        t += [(h + "ln_1.weight", [C]), (h + "ln_1.bias", [C]), (h + "attn.c_attn.weight", [C, 3 * C]),
              (h + "attn.c_attn.bias", [3 * C]), (h + "attn.c_proj.weight", [C, C]), (h + "attn.c_proj.bias", [C]),
              (h + "ln_2.weight", [C]), (h + "ln_2.bias", [C]), (h + "mlp.c_fc.weight", [C, FC]),
              (h + "mlp.c_fc.bias", [FC]), (h + "mlp.c_proj.weight", [FC, C]), (h + "mlp.c_proj.bias", [C])]
    return t


def _mix64(x):
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


def _values(seed, index, start, n):
    """float32 values start..start+n-1 of tensor `index`'s stream."""
    with np.errstate(over="ignore"):
        key = np.uint64((seed * 0x100000001B3 + index * 0x9E3779B1 + 1) & 0xFFFFFFFFFFFFFFFF)
        z = (np.arange(start, start + n, dtype=np.uint64) + key) * GOLD
        z ^= z >> np.uint64(30)
        z *= M1
        z ^= z >> np.uint64(27)
        z *= M2
        z ^= z >> np.uint64(31)
    u = (z >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / (1 << 24))
    return (u * np.float32(0.1) - np.float32(0.05)).astype(np.float32)


def write(path, tensors, dtype, seed, threads=8):
    """Write a safetensors file holding `tensors` [(name, shape)] in `dtype`
    ('BF16', 'F16' or 'F32').  BF16 keeps the top half of each FP32 value;
    F16 rounds it to nearest even."""
    esz = 4 if dtype == "F32" else 2
    order = sorted(range(len(tensors)), key=lambda i: _mix64(seed * 7919 + i))  # storage order
    header, off = {}, 0
    for i in order:
        name, shape = tensors[i]
        n = int(np.prod(shape))
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + n * esz]}
        off += n * esz
    header["__metadata__"] = {"format": "pt"}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.truncate(8 + len(hb) + off)
    data = np.memmap(path, dtype=np.uint8, mode="r+", offset=8 + len(hb), shape=(off,))

    jobs = []
    for i, (name, shape) in enumerate(tensors):
        a, b = header[name]["data_offsets"]
        n = (b - a) // esz
        for s in range(0, n, BLOCK):
            jobs.append((i, a, s, min(BLOCK, n - s)))

    def fill(job):
        i, a, s, n = job
        v = _values(seed, i, s, n)
        if dtype == "BF16":
            data[a + 2 * s:a + 2 * (s + n)] = (v.view(np.uint32) >> np.uint32(16)).astype(np.uint16).view(np.uint8)
        elif dtype == "F16":
            data[a + 2 * s:a + 2 * (s + n)] = v.astype(np.float16).view(np.uint8)
        else:
            data[a + 4 * s:a + 4 * (s + n)] = v.view(np.uint8)

    with ThreadPoolExecutor(threads) as pool:
        for _ in pool.map(fill, jobs):
            pass
    data.flush()
    del data
    return 8 + len(hb) + off


def write_qwen(path, seed):
    return write(path, qwen_tensors(), "BF16", seed)


def write_gpt2(path, seed):
    return write(path, gpt2_tensors(), "F32", seed)
