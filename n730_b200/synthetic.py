"""Seeded synthetic Qwen2-shape models (random-init weights ~ N(0, 0.02)).

There is no network in the build and benchmark environments, so models are
generated: HF tensor names, the shapes of Qwen2-0.5B / 7B / 72B, weights
N(0, 0.02), q/k/v biases N(0, 0.02), norms of ones.  Precision maps follow
the benchmark configurations:

* ``mixed_05b``   attention projections INT8 (reference per-tensor format),
                  FFN INT4 g128, embeddings / tied lm_head FP16;
* ``int4_g128``   every linear incl. embeddings and lm_head INT4 g128;
* ``aggressive``  FFN INT2 g64, attention INT4 g128, lm_head INT8 per channel,
                  embeddings INT4 g128.

Two builders: ``host_tensors`` (numpy, for files and oracle checks) and
``build_on_device`` (tensors drawn and quantised on the GPU with the
library's group quantiser, for full-size benchmarks).
"""
from __future__ import annotations

import numpy as np

from .engine import (BIAS_SLOTS, PROJ_SLOTS, V_FINAL_NORM, W_EMBED, W_LMHEAD, Engine, ModelShape,
                     qweight_from_device, qweight_from_block)

SHAPES = {
    "qwen2-0.5b": ModelShape(896, 24, 14, 2, 64, 4864, 151936, 1e6, 1e-6, True),
    "qwen2-7b": ModelShape(3584, 28, 28, 4, 128, 18944, 152064, 1e6, 1e-6, False),
    "qwen2-72b": ModelShape(8192, 80, 64, 8, 128, 29568, 152064, 1e6, 1e-6, False),
    "tiny": ModelShape(256, 2, 4, 2, 64, 512, 1000, 1e6, 1e-6, False),
    "tiny-gqa7": ModelShape(896, 2, 14, 2, 64, 1024, 2048, 1e6, 1e-6, True),
    "tiny-128": ModelShape(512, 2, 8, 2, 128, 1024, 1500, 1e6, 1e-6, False),
}


def precision_map(name: str):
    """Return f(tensor_name) -> assigned precision string (converter syntax)."""
    def mixed_05b(t):
        if t in ("model.embed_tokens.weight", "lm_head.weight"):
            return "FP16"
        return "INT8" if ".self_attn." in t else "INT4G128"

    def int4(t):
        return "INT4G128"

    def aggressive(t):
        if t == "lm_head.weight":
            return "INT8PC"
        if ".mlp." in t:
            return "INT2G64"
        return "INT4G128"

    return {"mixed_05b": mixed_05b, "int4_g128": int4, "aggressive": aggressive}[name]


def tensor_names(shape: ModelShape, biases: bool = True):
    """(name, shape) in HF order; 1-D entries are the q/k/v biases."""
    h, q, kv, f = shape.hidden, shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim, shape.ffn
    out = [("model.embed_tokens.weight", (shape.vocab, h))]
    for i in range(shape.layers):
        p = f"model.layers.{i}"
        out += [(f"{p}.self_attn.q_proj.weight", (q, h))]
        if biases:
            out += [(f"{p}.self_attn.q_proj.bias", (q,))]
        out += [(f"{p}.self_attn.k_proj.weight", (kv, h))]
        if biases:
            out += [(f"{p}.self_attn.k_proj.bias", (kv,))]
        out += [(f"{p}.self_attn.v_proj.weight", (kv, h))]
        if biases:
            out += [(f"{p}.self_attn.v_proj.bias", (kv,))]
        out += [(f"{p}.self_attn.o_proj.weight", (h, q)), (f"{p}.mlp.gate_proj.weight", (f, h)),
                (f"{p}.mlp.up_proj.weight", (f, h)), (f"{p}.mlp.down_proj.weight", (h, f))]
    if not shape.tie_embeddings:
        out.append(("lm_head.weight", (shape.vocab, h)))
    return out


def host_tensors(shape: ModelShape, seed: int = 0, std: float = 0.02, biases: bool = True):
    """Yield (name, fp32 array); each tensor drawn from default_rng(seed + index)."""
    for i, (name, shp) in enumerate(tensor_names(shape, biases)):
        rng = np.random.default_rng(seed * 100003 + i)
        yield name, rng.normal(0, std, shp).astype(np.float32)


def sensitivity_map(shape: ModelShape, pmap: str, biases: bool = True) -> dict:
    f = precision_map(pmap)
    names = tensor_names(shape, biases)
    profiles = [{"layer_name": n, "assigned_precision": f(n)} for n, s in names if len(s) == 2]
    return {"model_id": f"synthetic-{pmap}", "total_params": int(sum(np.prod(s) for _, s in names)),
            "total_layers": len(names), "profiles": profiles}


def write_n730(path, shape: ModelShape, pmap: str, seed: int = 0, biases: bool = True):
    from .converter import convert
    return convert(host_tensors(shape, seed, biases=biases), sensitivity_map(shape, pmap, biases), path,
                   verbose=False)


def build_on_device(shape: ModelShape, pmap: str, engine: Engine, seed: int = 0, std: float = 0.02,
                    biases: bool = True, tp_rank: int = 0, tp_size: int = 1, export=None):
    """Draw every tensor on the GPU and quantise it there; hand the packed weights
    to ``engine``.  Group-wise precisions use the library's GPU quantiser;
    per-tensor INT8 and FP16 (small tensors in the mixed map) are packed on
    the host by the converter's quantisers.  With ``tp_size > 1`` every rank
    draws the same full tensors and keeps its tensor-parallel shard
    (``n730_b200.tp.shard``); ``shape`` is the global shape.

    ``export(name, item)``, when given, receives a host copy of what the engine
    was handed for each tensor: ``{"kind": "grouped", "bits", "group", "rows",
    "cols", "codes", "s16", "z16"}`` (numpy), ``{"kind": "block", "block":
    RawBlock}`` for per-tensor formats, or ``{"kind": "vector", "v": fp32}`` for
    biases - so a checker can dequantise exactly the codes the engine runs."""
    from . import tp as tpmod
    import ctypes as C

    import torch

    from . import _lib
    from .converter import QUANTIZERS, parse_precision, serialize_layer
    from .formats import read_block, RawBlock
    lib = _lib.cuda()
    f = precision_map(pmap)
    stream = torch.cuda.current_stream().cuda_stream
    ffn_group = tpmod.ffn_group_of(f, "model.layers.0.mlp.down_proj.weight")
    for i, (name, shp) in enumerate(tensor_names(shape, biases)):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed * 100003 + i)
        w = torch.randn(shp, generator=g, device="cuda", dtype=torch.float32) * std
        if tp_size > 1:
            w = tpmod.shard(name, w, shape, tp_size, tp_rank, ffn_group)
            if w is None:
                continue
            w = w.contiguous()
            shp = tuple(w.shape)
        if len(shp) == 1:
            layer = int(name.split(".")[2])
            base = name.split(".", 3)[3].rsplit(".", 1)[0]
            v = w.cpu().numpy()
            engine.set_vector(layer, BIAS_SLOTS[base], v)
            if export:
                export(name, {"kind": "vector", "v": v})
            continue
        prec, group = parse_precision(f(name), {}, shp[1])
        if prec in ("INT2G", "INT4G", "INT8G"):
            bits = {"INT2G": 2, "INT4G": 4, "INT8G": 8}[prec]
            rows, cols = shp
            codes = torch.empty(rows * cols * bits // 8, dtype=torch.uint8, device="cuda")
            s16 = torch.empty(rows, cols // group, dtype=torch.float16, device="cuda")
            z16 = torch.empty_like(s16)
            _lib.check(lib.n730_quantize_grouped(C.c_void_p(w.data_ptr()), rows, cols, bits, group,
                                                 C.c_void_p(codes.data_ptr()), C.c_void_p(s16.data_ptr()),
                                                 C.c_void_p(z16.data_ptr()), C.c_void_p(stream)), "quantize")
            qw = qweight_from_device(0x40 | bits, rows, cols, group, codes.data_ptr(), s16.data_ptr(),
                                     z16.data_ptr(), stream=stream)
            torch.cuda.current_stream().synchronize()
            if export:
                export(name, {"kind": "grouped", "bits": bits, "group": group, "rows": rows, "cols": cols,
                              "codes": codes.cpu().numpy().reshape(rows, -1), "s16": s16.cpu().numpy(),
                              "z16": z16.cpu().numpy()})
            del codes, s16, z16
        else:
            block, _ = serialize_layer(0, prec, w.cpu().numpy(), name)
            import io
            import struct
            _, _, pid, r, c, sc, zp, dsz = struct.unpack(">4sIBIIffi", block[:29])
            rb = RawBlock(0, pid, r, c, sc, zp, block[29:29 + dsz], 0)
            qw = qweight_from_block(rb)
            if export:
                export(name, {"kind": "block", "block": rb})
        del w
        if name == "model.embed_tokens.weight":
            engine.set_qweight(-1, W_EMBED, qw)
        elif name == "lm_head.weight":
            engine.set_qweight(-1, W_LMHEAD, qw)
        else:
            layer = int(name.split(".")[2])
            base = name.split(".", 3)[3].rsplit(".", 1)[0]
            engine.set_qweight(layer, PROJ_SLOTS[base], qw)
    torch.cuda.synchronize()
