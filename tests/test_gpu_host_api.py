"""The reference-shaped host API (N730CudaTransformer, N730Generator) on the GPU engine."""
import numpy as np
import pytest

from gpu_util import rel_err
from oracle.model import OracleDecoder
from test_gpu_model import _blocks, _oracle_weights
from n730_b200 import synthetic
from n730_b200.inference import ModelConfig, N730CudaTransformer, N730Generator

pytestmark = pytest.mark.gpu


def _cfg(shape):
    c = ModelConfig()
    c.hidden_size, c.num_hidden_layers = shape.hidden, shape.layers
    c.num_attention_heads, c.num_kv_heads, c.head_dim = shape.heads, shape.kv_heads, shape.head_dim
    c.intermediate_size, c.vocab_size = shape.ffn, shape.vocab
    c.rope_theta, c.rms_norm_eps, c.max_position_embeddings = shape.rope_theta, shape.rms_eps, 512
    return c


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    shape = synthetic.SHAPES["tiny-gqa7"]
    path = tmp_path_factory.mktemp("h") / "tiny.n730"
    synthetic.write_n730(path, shape, "int4_g128", seed=9)
    return shape, str(path), _oracle_weights(_blocks(path))


def test_transformer_forward_and_kv(tiny):
    shape, path, w = tiny
    t = N730CudaTransformer(path, None, _cfg(shape), verbose=False)
    orc = OracleDecoder(shape, w, max_pos=512)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, shape.vocab, 33)
    assert rel_err(t.forward(prompt), orc.forward(prompt)) <= 1e-2
    tok = 7
    for _ in range(5):
        y, yr = t.forward([tok]), orc.forward([tok])
        assert y.shape == (shape.vocab,) and y.dtype == np.float32
        assert rel_err(y, yr) <= 1e-2
        tok = int(np.argmax(yr))
    assert t.kv.seq_len == 38
    t.kv.clear()
    assert t.kv.seq_len == 0
    orc2 = OracleDecoder(shape, w, max_pos=512)
    assert rel_err(t.forward([1, 2, 3]), orc2.forward([1, 2, 3])) <= 1e-2
    t.close()


def test_missing_tensor_is_rejected(tiny, tmp_path):
    shape, _, _ = tiny
    small = synthetic.SHAPES["tiny"]
    p = tmp_path / "other.n730"
    synthetic.write_n730(p, small, "int4_g128", seed=1)
    cfg = _cfg(small)
    cfg.num_hidden_layers = small.layers + 1  # the file has one layer fewer
    with pytest.raises(ValueError, match="missing"):
        N730CudaTransformer(str(p), None, cfg, verbose=False)


class _Tok:
    eos = -1

    def encode_chat(self, prompt):
        return np.array([ord(c) % 2048 for c in prompt], np.int32)

    def decode(self, ids):
        return " ".join(map(str, ids))


def test_generator_greedy_matches_oracle(tiny):
    shape, path, w = tiny
    gen = N730Generator.__new__(N730Generator)
    gen.cfg = _cfg(shape)
    gen.transformer = N730CudaTransformer(path, None, gen.cfg, verbose=False)
    gen.tok, gen.verbose, gen.last_stats = _Tok(), False, {}
    out = gen.generate("hello b200", max_tokens=6, temp=0)
    orc = OracleDecoder(shape, w, max_pos=512)
    want = [int(np.argmax(orc.forward(_Tok().encode_chat("hello b200"))))]
    for _ in range(5):
        want.append(int(np.argmax(orc.forward([want[-1]]))))
    assert out == want
    assert gen.last_stats["tokens"] == 6
    gen.transformer.close()
