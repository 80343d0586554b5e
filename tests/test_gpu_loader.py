"""Native .n730 block loader (n730_qweight_load_blocks, engine.load_file) against the
Python block reader (formats.read_block + qweight_from_block).

* every weight of files in the three precision maps (INT4 g128; INT8 per-tensor
  attention + FP16 tied embedding; INT2 g64 FFN + INT8 per-channel lm_head)
  dequantises bit-identically through both loaders, and an engine loaded either
  way gives identical logits;
* a Qwen2-72B-width layer (hidden 8192, FFN 29568) written by the streaming
  writer (converter.N730Writer) loads natively and decodes within the 1e-2
  bar of the oracle;
* bad offsets are rejected before any device work, leaving no handle behind.
"""
import ctypes as C
import dataclasses

import numpy as np
import pytest

from gpu_util import rel_err
from oracle.model import OracleDecoder
from test_gpu_model import _blocks, _oracle_weights
from n730_b200 import _lib, synthetic
from n730_b200.converter import N730Writer, parse_precision
from n730_b200.engine import Engine, _weight_slot, load_file, load_tensors, qweight_from_block, qweights_from_file
from n730_b200.formats import read_header

pytestmark = pytest.mark.gpu


def _dequant(qw):
    import torch
    lib = _lib.cuda()
    info = (C.c_int64 * 8)()
    _lib.check(lib.n730_qweight_info(qw, info), "info")
    out = torch.empty(info[2] * info[3], device="cuda")
    _lib.check(lib.n730_dequant_to_f32(qw, C.c_void_p(out.data_ptr()), None), "dequant")
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("shape_name,pmap", [("tiny", "int4_g128"), ("tiny-gqa7", "mixed_05b"),
                                             ("tiny-128", "aggressive")])
def test_native_blocks_match_python_reader(tmp_path, shape_name, pmap):
    shape = synthetic.SHAPES[shape_name]
    path = tmp_path / "m.n730"
    synthetic.write_n730(path, shape, pmap, seed=13)
    entries = [e for e in read_header(path)["seek_table"] if _weight_slot(e["layer_name"])]
    handles, nbytes = qweights_from_file(path, [e["file_offset"] for e in entries])
    assert nbytes == sum(29 + e["stored_bytes"] for e in entries)
    blocks = dict(_blocks(path))
    lib = _lib.cuda()
    for e, h in zip(entries, handles):
        ref = qweight_from_block(blocks[e["layer_name"]])
        assert np.array_equal(_dequant(h), _dequant(ref)), e["layer_name"]
        lib.n730_qweight_destroy(h)
        lib.n730_qweight_destroy(ref)
    # whole engines: native loader vs the Python reader
    ea = Engine(shape, max_ctx=128, max_batch=1, max_prefill=64)
    stats = load_file(ea, path)
    ea.finalize()
    assert stats["native_blocks"] == len(entries)
    eb = Engine(shape, max_ctx=128, max_batch=1, max_prefill=64)
    load_tensors(eb, _blocks(path))
    eb.finalize()
    prompt = np.arange(20) * 7 % shape.vocab
    assert np.array_equal(ea.forward(prompt), eb.forward(prompt))
    assert np.array_equal(ea.forward([3]), eb.forward([3]))
    ea.close()
    eb.close()


def test_72b_width_streamed_file_loads_natively(tmp_path):
    shape = dataclasses.replace(synthetic.SHAPES["qwen2-72b"], layers=1, vocab=4096)
    path = tmp_path / "w72.n730"
    names = synthetic.tensor_names(shape)
    f = synthetic.precision_map("int4_g128")
    wr = N730Writer(path, "synthetic-72b-width", sum(int(np.prod(s)) for _, s in names), len(names))
    for name, w in synthetic.host_tensors(shape, seed=17):
        prec, group = parse_precision(f(name), {}, w.shape[-1]) if w.ndim == 2 else ("FP16", 0)
        wr.add(name, w, prec, group)
        del w
    wr.close()
    e = Engine(shape, max_ctx=256, max_batch=1, max_prefill=256)
    stats = load_file(e, path)
    e.finalize()
    assert stats["python_blocks"] == 3 and stats["native_blocks"] == 9  # q/k/v biases in Python
    assert e.info()["persistent_decode"] and e.info()["ffn_fused"]
    orc = OracleDecoder(shape, _oracle_weights(_blocks(path)), max_pos=256)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, shape.vocab, 150)
    assert rel_err(e.forward(prompt), orc.forward(prompt)) <= 1e-2
    tok = 5
    for _ in range(4):
        y, yr = e.forward([tok]), orc.forward([tok])
        assert rel_err(y, yr) <= 1e-2
        tok = int(np.argmax(yr))
    e.close()


def test_bad_offsets_rejected(tmp_path):
    shape = synthetic.SHAPES["tiny"]
    path = tmp_path / "m.n730"
    synthetic.write_n730(path, shape, "int4_g128", seed=2)
    good = [e["file_offset"] for e in read_header(path)["seek_table"]][:2]
    with pytest.raises(_lib.N730Error):
        qweights_from_file(path, good + [good[1] + 13])  # not a block header
    with pytest.raises(_lib.N730Error):
        qweights_from_file(path, good + [10 ** 12])  # past the end
    with pytest.raises(_lib.N730Error):
        qweights_from_file(tmp_path / "missing.n730", good)
