"""Inference host API: the reference's ``src-code/inference.py`` surface on this build.

Same names and semantics as the reference (``ModelConfig``, ``DeviceBuf``,
``VRAMKVCache``, ``N730CudaTransformer.forward(token_ids) -> logits``,
``sample``, ``Tokenizer``, ``N730Generator.generate``; ``inference.py:145-772``),
but ``forward`` is one call into the resident whole-model engine
(``n730_model_forward``): packed weights are uploaded once, every linear is a
fused dequant-GEMV, attention runs over a paged fp16 KV cache, and the final
norm + lm_head run on the GPU.  Returns float32 logits of the last position,
like the reference (``inference.py:648-669``).
"""
from __future__ import annotations

import ctypes as C
import json
import time
from pathlib import Path
from typing import Dict, Optional

import numpy as np

from . import _lib, model_compat
from .engine import Engine, ModelShape, load_file, load_tensors
from .formats import read_block, read_header
from .scheduler import N730Scheduler


def check(rc, what: str = ""):
    """Raise on a negative return code (``inference.py:141-143``)."""
    return _lib.check(rc, what)


class ModelConfig:
    """HF-style config with the reference's defaults and field names (``inference.py:145-208``)."""

    def __init__(self, path=None, hf_path=None):
        self.hidden_size = 1536
        self.num_hidden_layers = 28
        self.num_attention_heads = 12
        self.num_kv_heads = 2
        self.head_dim = 128
        self.intermediate_size = 8960
        self.vocab_size = 151936
        self.rms_norm_eps = 1e-6
        self.rope_theta = 10000.0
        self.max_position_embeddings = 131072
        self.tie_word_embeddings = False
        self.compat = None
        if path and Path(path).exists():
            self._apply(json.loads(Path(path).read_text()))
        if hf_path:
            cfg = None
            local = Path(hf_path) / "config.json"
            if local.exists():
                cfg = json.loads(local.read_text())
            else:
                try:
                    from huggingface_hub import hf_hub_download
                    cfg = json.loads(Path(hf_hub_download(repo_id=hf_path, filename="config.json")).read_text())
                except Exception as e:
                    print(f"  WARNING: no config.json for {hf_path!r} ({e}); keeping built-in defaults")
            if cfg is not None:
                self._apply(cfg)
                self.compat = model_compat.check(cfg)
                if not self.compat.ok:
                    print(f"  WARNING: {self.compat.architecture} is not supported: " + "; ".join(self.compat.reasons))

    def _apply(self, c: dict):
        self.hidden_size = c.get("hidden_size", self.hidden_size)
        self.num_hidden_layers = c.get("num_hidden_layers", self.num_hidden_layers)
        self.num_attention_heads = c.get("num_attention_heads", self.num_attention_heads)
        self.num_kv_heads = c.get("num_key_value_heads", self.num_kv_heads)
        self.intermediate_size = c.get("intermediate_size", self.intermediate_size)
        self.vocab_size = c.get("vocab_size", self.vocab_size)
        self.rms_norm_eps = c.get("rms_norm_eps", self.rms_norm_eps)
        self.rope_theta = c.get("rope_theta", self.rope_theta)
        self.max_position_embeddings = c.get("max_position_embeddings", self.max_position_embeddings)
        self.tie_word_embeddings = c.get("tie_word_embeddings", self.tie_word_embeddings)
        self.head_dim = self.hidden_size // self.num_attention_heads

    def shape(self, tie_embeddings: Optional[bool] = None) -> ModelShape:
        return ModelShape(self.hidden_size, self.num_hidden_layers, self.num_attention_heads, self.num_kv_heads,
                          self.head_dim, self.intermediate_size, self.vocab_size, float(self.rope_theta),
                          float(self.rms_norm_eps),
                          self.tie_word_embeddings if tie_embeddings is None else tie_embeddings)


class DeviceBuf:
    """Owns a device allocation of n floats (``inference.py:210-228``)."""

    def __init__(self, lib, n_floats: int):
        self._lib = lib
        self._ptr = C.c_void_p(0)
        check(lib.n730_device_alloc(n_floats, C.byref(self._ptr)), "device_alloc")
        self.n = n_floats

    @property
    def ptr(self):
        return self._ptr

    def fp(self):
        return C.cast(self._ptr, C.POINTER(C.c_float))

    def __del__(self):
        if getattr(self, "_ptr", None):
            self._lib.n730_device_free(self._ptr)
            self._ptr = C.c_void_p(0)


class VRAMKVCache:
    """The reference's KV-cache handle (``inference.py:230-257``) over the engine's
    paged fp16 cache: ``seq_len``, ``clear()``, ``vram_mb``."""

    def __init__(self, engine: Engine, seq: int = 0):
        self._engine = engine
        self._seq = seq

    @property
    def seq_len(self) -> int:
        return self._engine.seq_len(self._seq)

    @seq_len.setter
    def seq_len(self, n: int):
        self._engine.set_seq_len(self._seq, n)

    def clear(self):
        self._engine.set_seq_len(self._seq, 0)

    @property
    def max_seq(self) -> int:
        return self._engine.max_ctx

    @property
    def vram_mb(self) -> float:
        return self._engine.info()["kv_capacity_bytes"] / 2**20


def _load_hf_norms(hf_path: str) -> Dict[str, np.ndarray]:
    """Norm vectors from a local/Hub checkpoint via transformers, best effort (``inference.py:368-387``)."""
    try:
        import torch
        from transformers import AutoModelForCausalLM
        m = AutoModelForCausalLM.from_pretrained(hf_path, dtype=torch.float32, device_map="cpu",
                                                 low_cpu_mem_usage=True)
        out = {n: p.detach().numpy().astype(np.float32) for n, p in m.named_parameters()
               if "norm" in n.lower() and p.ndim == 1}
        del m
        return out
    except Exception as e:
        print(f"  norm load failed ({e}); identity norms")
        return {}


class N730CudaTransformer:
    """Resident-weight decoder over a ``.n730`` file (``inference.py:259-669``)."""

    def __init__(self, model_path: str, hf_path: Optional[str], cfg: ModelConfig, prefetch: int = 8,
                 max_ctx: Optional[int] = None, norms: Optional[Dict[str, np.ndarray]] = None,
                 verbose: bool = True, **engine_kw):
        self.cfg = cfg
        self.lib = _lib.cuda()
        self._sched = N730Scheduler(model_path, prefetch=prefetch, verbose=verbose)
        self._seek_table = self._sched._seek_table
        self._name_to_entry = {e["layer_name"]: e for e in self._seek_table}
        self._validate_model_layout()
        tied = "lm_head.weight" not in self._name_to_entry
        self.norm_w = dict(norms or {})
        if not self.norm_w and hf_path:
            self.norm_w = _load_hf_norms(hf_path)
        max_ctx = max_ctx or min(int(cfg.max_position_embeddings), 4096)
        self.engine = Engine(cfg.shape(tie_embeddings=tied), max_ctx=max_ctx, **engine_kw)
        # 2-D weights through the native block loader (pread into pinned staging, async copies)
        self.load_stats = load_file(self.engine, model_path, self.norm_w)
        self.engine.finalize()
        self.kv = VRAMKVCache(self.engine)
        if verbose:
            print(f"  {self.lib.n730_cuda_version().decode()}  weights {self.engine.info()['weight_bytes'] / 2**20:.1f}"
                  f" MB resident, KV {self.kv.vram_mb:.1f} MB ({max_ctx} positions)")

    def _validate_model_layout(self):
        """Every projection of every layer must be present (``inference.py:325-348``)."""
        need = ["model.embed_tokens.weight"]
        for i in range(self.cfg.num_hidden_layers):
            p = f"model.layers.{i}"
            need += [f"{p}.self_attn.{t}_proj.weight" for t in "qkvo"]
            need += [f"{p}.mlp.{t}_proj.weight" for t in ("gate", "up", "down")]
        missing = [n for n in need if n not in self._name_to_entry]
        if missing:
            more = " ..." if len(missing) > 4 else ""
            raise ValueError(f"Model file is missing {len(missing)} required tensors: {', '.join(missing[:4])}{more}")

    def forward(self, token_ids) -> np.ndarray:
        """Append ``token_ids`` to the sequence; float32 logits of the last position."""
        return self.engine.forward(np.asarray(token_ids, np.int32), seq=0)

    def forward_sample(self, token: int, temp: float = 0.7, top_p: float = 0.9, seed: int = 0) -> int:
        """Append one token and sample the next on the GPU (``n730_sample``): only the token id
        crosses back to the host, not the logits."""
        return int(self.engine.decode_sample([token], temp, top_p, seed)[0])

    def close(self):
        self.engine.close()


def sample(logits: np.ndarray, temp: float = 0.7, top_p: float = 0.9, rng=None) -> int:
    """Temperature + nucleus sampling (``inference.py:674-682``); temp <= 0 is argmax."""
    if temp <= 0:
        return int(np.argmax(logits))
    z = (logits.astype(np.float32) - logits.max()) / temp
    p = np.exp(z)
    p /= p.sum()
    order = np.argsort(p)[::-1]
    keep = int(np.searchsorted(np.cumsum(p[order]), top_p)) + 1
    idx = order[:keep]
    q = p[idx] / p[idx].sum()
    return int((rng or np.random).choice(idx, p=q))


class Tokenizer:
    """HF tokenizer wrapper (``inference.py:684-709``)."""

    def __init__(self, path):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, trust_remote_code=True)
        self.eos = self.tok.eos_token_id

    def encode(self, text):
        return np.array(self.tok.encode(text), np.int32)

    def encode_chat(self, prompt):
        if getattr(self.tok, "chat_template", None):
            ids = self.tok.apply_chat_template([{"role": "user", "content": prompt}], tokenize=True,
                                               add_generation_prompt=True)
            if hasattr(ids, "get") and ids.get("input_ids") is not None:
                ids = ids["input_ids"]
            if hasattr(ids, "tolist"):
                ids = ids.tolist()
            if ids and isinstance(ids[0], (list, tuple)):
                ids = ids[0]
            return np.asarray(ids, np.int32)
        return self.encode(prompt)

    def decode(self, ids):
        return self.tok.decode(list(ids), skip_special_tokens=False)


class N730Generator:
    """Prompt in, tokens out (``inference.py:711-745``).  ``tokenizer`` may be any
    object with ``encode_chat``, ``decode`` and ``eos`` (default: the HF
    tokenizer of ``hf_path``)."""

    def __init__(self, model_path, hf_path=None, config_path=None, prefetch=8, tokenizer=None, verbose=True,
                 **kw):
        self.cfg = ModelConfig(config_path, hf_path=hf_path)
        self.transformer = N730CudaTransformer(model_path, hf_path, self.cfg, prefetch, verbose=verbose, **kw)
        self.tok = tokenizer if tokenizer is not None else Tokenizer(hf_path)
        self.verbose = verbose
        self.last_stats = {}

    def generate(self, prompt, max_tokens=200, temp=0.7, top_p=0.9, rng=None, gpu_sampling=True):
        """With ``gpu_sampling`` (default) every decode step samples on the GPU (the draws are
        seeded from ``rng``, or at random); ``gpu_sampling=False`` samples the logits on the host
        with ``sample`` (reproducible with a numpy ``rng``)."""
        self.transformer.kv.clear()
        ids = self.tok.encode_chat(prompt)
        t0 = time.perf_counter()
        tok = sample(self.transformer.forward(ids), temp, top_p, rng)
        out = [tok]
        prefill_s = time.perf_counter() - t0
        seed = int(rng.integers(0, 2**62)) if hasattr(rng, "integers") else int(np.random.randint(0, 2**31))
        t1 = time.perf_counter()
        while len(out) < max_tokens and tok != self.tok.eos:
            if gpu_sampling:
                tok = self.transformer.forward_sample(tok, temp, top_p, seed)
            else:
                tok = sample(self.transformer.forward([tok]), temp, top_p, rng)
            out.append(tok)
        n = max(len(out) - 1, 1)
        tps = n / max(time.perf_counter() - t1, 1e-6)
        self.last_stats = {"tokens": len(out), "prefill_s": prefill_s, "tok_per_s": tps}
        if self.verbose:
            print(f"  {self.tok.decode(out)}\n  [{len(out)} tokens | prefill {prefill_s:.2f}s | {tps:.1f} tok/s]")
        return out
