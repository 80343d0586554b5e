"""Host-side mirror of the reference's inference/scheduler/model_compat APIs (no GPU)."""
import json

import numpy as np
import pytest

from conftest import GOLDEN
from n730_b200 import model_compat
from n730_b200.formats import read_header
from n730_b200.inference import ModelConfig, sample
from n730_b200.scheduler import LayerBuffer, N730Scheduler, SchedulerStats


@pytest.fixture(scope="module")
def built():
    from n730_b200 import build
    build.build()


def test_compat_supported_and_blocked():
    ok = model_compat.check({"architectures": ["Qwen2ForCausalLM"], "hidden_size": 3584, "num_attention_heads": 28,
                             "tie_word_embeddings": True, "sliding_window": 4096})
    assert ok.ok and ok.architecture == "Qwen2ForCausalLM" and len(ok.warnings) == 2
    bad = model_compat.check({"architectures": ["MixtralForCausalLM"]})
    assert not bad.ok and "mixture-of-experts" in bad.reasons[0]
    for cfg, key in [({"hidden_act": "gelu"}, "hidden_act"), ({"rope_interleaved": True}, "rope_interleaved"),
                     ({"partial_rotary_factor": 0.5}, "partial_rotary"), ({"num_experts": 8}, "mixture"),
                     ({"hidden_size": 4096, "num_attention_heads": 32, "head_dim": 256}, "head_dim")]:
        r = model_compat.check({"architectures": ["LlamaForCausalLM"], **cfg})
        assert not r.ok and any(key in x for x in r.reasons), cfg
    assert "compatible: NO" in bad.describe()


def test_compat_repo(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"architectures": ["MistralForCausalLM"]}))
    assert model_compat.check_repo(str(tmp_path)).ok


def test_model_config_from_hf_dir(tmp_path):
    cfg = {"architectures": ["Qwen2ForCausalLM"], "hidden_size": 896, "num_hidden_layers": 24,
           "num_attention_heads": 14, "num_key_value_heads": 2, "intermediate_size": 4864, "vocab_size": 151936,
           "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "max_position_embeddings": 32768,
           "tie_word_embeddings": True}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    c = ModelConfig(hf_path=str(tmp_path))
    assert (c.hidden_size, c.num_kv_heads, c.head_dim, c.rope_theta) == (896, 2, 64, 1e6)
    assert c.compat.ok
    s = c.shape()
    assert (s.hidden, s.layers, s.heads, s.kv_heads, s.ffn, s.tie_embeddings) == (896, 24, 14, 2, 4864, True)
    d = ModelConfig()  # the reference's defaults
    assert (d.hidden_size, d.num_hidden_layers, d.rope_theta) == (1536, 28, 10000.0)


def test_sample():
    logits = np.array([0.1, 3.0, -1.0, 2.9], np.float32)
    assert sample(logits, temp=0) == 1
    rng = np.random.default_rng(0)
    got = {sample(logits, temp=0.7, top_p=0.5, rng=rng) for _ in range(50)}
    assert got <= {1, 3}  # nucleus of mass 0.5 holds the two top tokens only
    assert sample(logits, temp=1.0, top_p=1e-6, rng=rng) == 1


def test_scheduler_stream_and_get_layer(built, golden):
    s = N730Scheduler(str(GOLDEN / "ref_small.n730"), prefetch=2, verbose=False)
    hdr = read_header(GOLDEN / "ref_small.n730")
    seen = []
    for layer in s.stream():
        assert isinstance(layer, LayerBuffer)
        k = layer.layer_name.replace(".", "_")
        ref = golden[k + "__n730core"].reshape(layer.weights.shape)
        assert np.array_equal(layer.weights.view(np.uint32), ref.view(np.uint32)), layer.layer_name
        seen.append(layer.layer_idx)
    assert seen == [e["layer_idx"] for e in hdr["seek_table"]]
    st = s.stats
    assert isinstance(st, SchedulerStats) and st.total_layers == len(seen)
    assert st.total_bytes_read == sum(e["stored_bytes"] for e in hdr["seek_table"])
    assert st.prefetch_hits + st.prefetch_misses == len(seen) and 0 <= st.hit_rate <= 1
    one = s.get_layer(3)
    k = one.layer_name.replace(".", "_")
    assert np.array_equal(one.weights.reshape(-1).view(np.uint32), golden[k + "__n730core"].reshape(-1).view(np.uint32))
    part = [l.layer_idx for l in s.stream(2, 5)]
    assert part == [e["layer_idx"] for e in hdr["seek_table"][2:5]]
    s.close()


def test_scheduler_rejects_bad_file(built, tmp_path):
    bad = tmp_path / "bad.n730"
    bad.write_bytes(b"NOTN730!" + bytes(64))
    with pytest.raises(RuntimeError, match="BAD_MAGIC"):
        N730Scheduler(str(bad), verbose=False)
