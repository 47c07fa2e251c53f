"""Checkpoint converters: Hugging Face safetensors -> the engines' flat weight files.

The two output formats are the ones the decode engines load (and the
reference engines too: qwen_engine.c:61-75, gpt2_engine.c:51-70):

* Qwen2.5-0.5B, FP16 (990,162,688 B), written by the reference's
  gpu-llm/tools/conv_qwen.py:63-99 -- embedding, FP32 RoPE cos/sin tables
  [8192][32], 24 layers of in_ln | qkv_w (q|k|v rows) | qkv_b | o_w |
  post_ln | gateup_w (gate rows, then up rows) | down_w, final norm.
  Linear weights are already [out, in]; BF16/F16/F32 sources are widened to
  FP32 exactly and rounded to FP16 once (round to nearest even, subnormals
  kept), as the reference does.
* GPT-2 124M, FP32 (124,439,808 floats), written by
  gpu-llm/tools/conv_gpt2.py:38-62 -- wte, wpe, 12 layers of ln_1 w/b |
  c_attn w/b | attn c_proj w/b | ln_2 w/b | c_fc w/b | mlp c_proj w/b,
  ln_f w/b.  Conv1D weights are stored [in, out] by Hugging Face and are
  transposed to [out, in].  The source must be F32 (conv_gpt2.py:23).

Both produce files byte-identical to the reference converters' on the same
checkpoint.  Unlike the reference scripts (one sequential pass holding
whole tensors), the output is a memory-mapped file filled by a thread pool,
one task per weight segment, with large tensors converted in bounded row
chunks; the source is memory-mapped, so nothing is read twice.

CLI, with the reference scripts' defaults:
    python sb_convert.py qwen [model.safetensors] [qwen_05b.bin]
    python sb_convert.py gpt2 [model.safetensors] [gpt2_124m.bin]
"""
import json
import os
import struct
import sys
from concurrent.futures import ThreadPoolExecutor

import numpy as np

QWEN = dict(V=151936, C=896, NL=24, NH=14, NKV=2, HD=64, FC=4864, CTX=8192, THETA=1_000_000.0,
            FILE_BYTES=990162688)
GPT2 = dict(V=50257, C=768, NL=12, FC=3072, CTX=1024, TOTAL_FLOATS=124439808)

CHUNK_ELEMS = 1 << 23  # rows per conversion step are chosen to stay near 8 Mi elements


class ConvertError(ValueError):
    pass


class SafeTensors:
    """Read-only view of a .safetensors file: 8-byte little-endian header size,
    a JSON header {name: {dtype, shape, data_offsets}}, then the raw data."""

    _DT = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}

    def __init__(self, path):
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            self.header = json.loads(f.read(n).decode("utf-8"))
        self.header.pop("__metadata__", None)
        self._raw = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)

    def __contains__(self, name):
        return name in self.header

    def shape(self, name):
        return list(self.header[name]["shape"])

    def dtype(self, name):
        return self.header[name]["dtype"]

    def raw(self, name):
        """The tensor in its stored dtype (BF16 as uint16 bit patterns), zero-copy."""
        m = self.header[name]
        dt = self._DT.get(m["dtype"])
        if dt is None:
            raise ConvertError(f"unsupported dtype {m['dtype']} for {name}")
        a, b = m["data_offsets"]
        return self._raw[a:b].view(dt).reshape(m["shape"])


def widen(a):
    """Stored values -> FP32, exactly (BF16 bit patterns shift into the high half)."""
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def _rows_per_chunk(cols):
    return max(1, CHUNK_ELEMS // max(1, cols))


def qwen_plan(st):
    """(byte offset, element count, producer) segments of the Qwen file.  A
    producer writes its FP16 elements into the destination slice it gets."""
    q = QWEN
    V, C, NL, HD, FC = q["V"], q["C"], q["NL"], q["HD"], q["FC"]
    KVD = q["NKV"] * HD
    QKV = C + 2 * KVD
    want = {"model.embed_tokens.weight": [V, C], "model.norm.weight": [C]}
    for i in range(NL):
        p = f"model.layers.{i}."
        want.update({p + "input_layernorm.weight": [C], p + "post_attention_layernorm.weight": [C],
                     p + "self_attn.q_proj.weight": [C, C], p + "self_attn.k_proj.weight": [KVD, C],
                     p + "self_attn.v_proj.weight": [KVD, C], p + "self_attn.q_proj.bias": [C],
                     p + "self_attn.k_proj.bias": [KVD], p + "self_attn.v_proj.bias": [KVD],
                     p + "self_attn.o_proj.weight": [C, C], p + "mlp.gate_proj.weight": [FC, C],
                     p + "mlp.up_proj.weight": [FC, C], p + "mlp.down_proj.weight": [C, FC]})
    for name, shp in want.items():
        if name not in st:
            raise ConvertError(f"checkpoint has no tensor {name}")
        if st.shape(name) != shp:
            raise ConvertError(f"{name}: shape {st.shape(name)}, expected {shp}")

    def half(names):  # FP16 rows of one or more same-width tensors, stacked in order
        def produce(dst):
            at = 0
            for name in names:
                src = st.raw(name)
                rows = src.shape[0]
                src2 = src.reshape(rows, -1)
                cols = src2.shape[1]
                step = _rows_per_chunk(cols)
                for r0 in range(0, rows, step):
                    r1 = min(rows, r0 + step)
                    n = (r1 - r0) * cols
                    dst[at:at + n] = widen(src2[r0:r1]).astype(np.float16).reshape(-1)
                    at += n
        return produce

    def rope(which):  # the reference's table formula, in float64, stored as FP32
        def produce(dst):
            d = np.arange(HD // 2, dtype=np.float64)
            freq = q["THETA"] ** (-2.0 * d / HD)
            ang = np.outer(np.arange(q["CTX"], dtype=np.float64), freq)
            dst[:] = (np.cos(ang) if which == 0 else np.sin(ang)).astype(np.float32).reshape(-1)
        return produce

    segs, off = [], 0

    def add(nbytes, elem, produce):
        nonlocal off
        segs.append((off, nbytes // elem, elem, produce))
        off += nbytes

    add(V * C * 2, 2, half(["model.embed_tokens.weight"]))
    tab = q["CTX"] * (HD // 2) * 4
    add(tab, 4, rope(0))
    add(tab, 4, rope(1))
    for i in range(NL):
        p = f"model.layers.{i}."
        add(C * 2, 2, half([p + "input_layernorm.weight"]))
        add(QKV * C * 2, 2, half([p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                  p + "self_attn.v_proj.weight"]))
        add(QKV * 2, 2, half([p + "self_attn.q_proj.bias", p + "self_attn.k_proj.bias", p + "self_attn.v_proj.bias"]))
        add(C * C * 2, 2, half([p + "self_attn.o_proj.weight"]))
        add(C * 2, 2, half([p + "post_attention_layernorm.weight"]))
        add(2 * FC * C * 2, 2, half([p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"]))
        add(C * FC * 2, 2, half([p + "mlp.down_proj.weight"]))
    add(C * 2, 2, half(["model.norm.weight"]))
    if off != q["FILE_BYTES"]:
        raise ConvertError(f"internal layout error: {off} bytes planned, {q['FILE_BYTES']} expected")
    return segs, off


def gpt2_plan(st):
    """Segments of the GPT-2 file (FP32).  Hugging Face names may carry a
    'transformer.' prefix; both spellings are accepted."""
    g = GPT2
    V, C, NL, FC = g["V"], g["C"], g["NL"], g["FC"]

    def key(name):
        if name in st:
            return name
        if "transformer." + name in st:
            return "transformer." + name
        raise ConvertError(f"checkpoint has no tensor {name}")

    order = [("wte.weight", [V, C], False), ("wpe.weight", [g["CTX"], C], False)]
    for i in range(NL):
        h = f"h.{i}."
        order += [(h + "ln_1.weight", [C], False), (h + "ln_1.bias", [C], False),
                  (h + "attn.c_attn.weight", [C, 3 * C], True), (h + "attn.c_attn.bias", [3 * C], False),
                  (h + "attn.c_proj.weight", [C, C], True), (h + "attn.c_proj.bias", [C], False),
                  (h + "ln_2.weight", [C], False), (h + "ln_2.bias", [C], False),
                  (h + "mlp.c_fc.weight", [C, FC], True), (h + "mlp.c_fc.bias", [FC], False),
                  (h + "mlp.c_proj.weight", [FC, C], True), (h + "mlp.c_proj.bias", [C], False)]
    order += [("ln_f.weight", [C], False), ("ln_f.bias", [C], False)]

    segs, off = [], 0
    for name, shp, transpose in order:
        k = key(name)
        if st.shape(k) != shp:
            raise ConvertError(f"{k}: shape {st.shape(k)}, expected {shp}")
        if st.dtype(k) != "F32":
            raise ConvertError(f"{k}: dtype {st.dtype(k)}, the GPT-2 converter takes F32 only")
        n = int(np.prod(shp))

        def produce(dst, k=k, transpose=transpose):
            src = st.raw(k)
            if not transpose:
                dst[:] = src.reshape(-1)
                return
            # [in, out] -> [out, in]: a chunk of output rows is a column block of the source
            cols_in, rows_out = src.shape
            step = _rows_per_chunk(cols_in)
            for r0 in range(0, rows_out, step):
                r1 = min(rows_out, r0 + step)
                dst[r0 * cols_in:r1 * cols_in] = np.ascontiguousarray(src[:, r0:r1].T).reshape(-1)

        segs.append((off, n, 4, produce))
        off += n * 4
    if off != g["TOTAL_FLOATS"] * 4:
        raise ConvertError(f"internal layout error: {off // 4} floats planned, {g['TOTAL_FLOATS']} expected")
    return segs, off


PLANS = {"qwen": qwen_plan, "gpt2": gpt2_plan}


def convert(model, src, out, threads=None, log=None):
    """Convert checkpoint `src` into the engine file `out` for `model`
    ('qwen' or 'gpt2').  Returns the bytes written.  Every tensor is checked
    (presence, shape, dtype) before the output file is created."""
    if model not in PLANS:
        raise ConvertError(f"unknown model {model!r} (qwen or gpt2)")
    st = SafeTensors(src)
    segs, total = PLANS[model](st)
    tmp = out + ".partial"
    dst = np.memmap(tmp, dtype=np.uint8, mode="w+", shape=(total,))
    try:
        def run(seg):
            off, n, elem, produce = seg
            view = dst[off:off + n * elem].view(np.float16 if (model == "qwen" and elem == 2) else np.float32)
            produce(view)

        with ThreadPoolExecutor(max_workers=threads or min(16, os.cpu_count() or 1)) as pool:
            for _ in pool.map(run, segs):
                pass
        dst.flush()
    except BaseException:
        del dst
        os.unlink(tmp)
        raise
    del dst
    os.replace(tmp, out)
    if log:
        log(f"wrote {out}: {total} bytes ({total / 1048576:.1f} MiB), {len(segs)} segments")
    return total


def main(argv):
    defaults = {"qwen": ("weights/qwen/model.safetensors", "qwen_05b.bin"),
                "gpt2": ("weights/model.safetensors", "gpt2_124m.bin")}
    if len(argv) < 2 or argv[1] not in defaults:
        sys.stderr.write("usage: sb_convert.py {qwen|gpt2} [model.safetensors] [out.bin]\n")
        return 2
    model = argv[1]
    src = argv[2] if len(argv) > 2 else defaults[model][0]
    out = argv[3] if len(argv) > 3 else defaults[model][1]
    try:
        convert(model, src, out, log=print)
    except (ConvertError, OSError, KeyError) as exc:
        sys.stderr.write(f"conversion failed: {exc}\n")
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
