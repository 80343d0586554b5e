"""Architecture gate for HF configs: which checkpoints the engine computes correctly.

Mirror of the reference's ``src-code/model_compat.py`` (same names and result
type, ``check(config) -> CompatResult``, ``check_repo(path)``): the engine
implements the Llama/Qwen2/Mistral/StableLM block - RMSNorm, rotate_half RoPE
over the whole head, GQA attention, SwiGLU MLP, optional q/k/v biases
(``model_compat.py:8-13,46-98``).  Configs that need anything else get a hard
reason; behaviours that merely diverge get a warning (``:100-107``).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

SUPPORTED_ARCHITECTURES = {
    "LlamaForCausalLM",
    "Qwen2ForCausalLM",
    "MistralForCausalLM",
    "StableLmForCausalLM",
}

# why a few common families fall outside the supported block
KNOWN_INCOMPATIBLE_NOTES = {
    "MixtralForCausalLM": "mixture-of-experts MLP (expert routing is not implemented)",
    "Phi3ForCausalLM": "partial rotary embedding and a fused qkv projection",
    "GemmaForCausalLM": "GeGLU MLP and extra feed-forward norms",
    "Gemma2ForCausalLM": "GeGLU, logit soft-capping and alternating sliding/full attention",
    "FalconForCausalLM": "fused qkv and parallel attention/MLP blocks",
    "GPT2LMHeadModel": "LayerNorm and learned absolute positions instead of RMSNorm + RoPE",
    "GPTNeoXForCausalLM": "LayerNorm and interleaved rotary embedding",
}


@dataclass
class CompatResult:
    ok: bool
    architecture: str = "unknown"
    reasons: list = field(default_factory=list)    # blockers
    warnings: list = field(default_factory=list)   # runs, but diverges or is worth noting

    def describe(self) -> str:
        out = [f"architecture: {self.architecture}", f"compatible: {'yes' if self.ok else 'NO'}"]
        out += [f"  x {r}" for r in self.reasons]
        out += [f"  ! {w}" for w in self.warnings]
        return "\n".join(out)


def check(config: dict) -> CompatResult:
    archs = config.get("architectures") or []
    arch = archs[0] if archs else config.get("model_type", "unknown")
    res = CompatResult(ok=True, architecture=arch)

    def block(msg):
        res.ok = False
        res.reasons.append(msg)

    if arch not in SUPPORTED_ARCHITECTURES:
        msg = f"'{arch}' is outside the supported Llama/Qwen2/Mistral/StableLM family"
        if arch in KNOWN_INCOMPATIBLE_NOTES:
            msg += f": {KNOWN_INCOMPATIBLE_NOTES[arch]}"
        block(msg)
        return res

    act = config.get("hidden_act", "silu")
    if act not in ("silu", "swish"):
        block(f"hidden_act={act!r}: the MLP epilogue computes SwiGLU (silu) only")
    if config.get("rope_interleaved"):
        block("rope_interleaved=true: the kernels rotate pairs (i, i + head_dim/2) (rotate_half), not adjacent pairs")
    prf = config.get("partial_rotary_factor", 1.0)
    if prf != 1.0:
        block(f"partial_rotary_factor={prf}: RoPE is applied to the whole head")
    if config.get("num_local_experts") or config.get("num_experts"):
        block("mixture-of-experts config: expert routing is not implemented")
    hidden, heads, hd = config.get("hidden_size"), config.get("num_attention_heads"), config.get("head_dim")
    if hidden and heads and hd and hd != hidden // heads:
        block(f"head_dim={hd} differs from hidden_size // num_attention_heads = {hidden // heads}; "
              "the loader derives head_dim from hidden_size")

    if config.get("sliding_window"):
        res.warnings.append(f"sliding_window={config['sliding_window']}: attention here is full (not windowed); "
                            "outputs diverge past the window")
    if config.get("tie_word_embeddings"):
        res.warnings.append("tie_word_embeddings=true: the lm_head reads the embedding matrix")
    return res


def check_repo(repo_id_or_path: str) -> CompatResult:
    """check() on ``<dir>/config.json``, or on a Hub repo's config when online."""
    local = Path(repo_id_or_path) / "config.json"
    if local.exists():
        return check(json.loads(local.read_text()))
    from huggingface_hub import hf_hub_download  # no network: raises, as the reference would
    return check(json.loads(Path(hf_hub_download(repo_id=repo_id_or_path, filename="config.json")).read_text()))
