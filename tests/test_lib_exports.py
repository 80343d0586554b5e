"""The C-ABI libraries load on a CPU host and export every declared symbol."""
import re
import subprocess

import pytest

from conftest import REPO

HEADERS = {"n730_cuda.so": REPO / "include" / "n730_cuda.h",
           "n730core.so": REPO / "include" / "n730core.h"}


def _declared(header):
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(n730_[a-z0-9_]+)\s*\(", text)))


def _exported(so):
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True,
                         check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


@pytest.fixture(scope="module", autouse=True)
def built():
    from n730_b200 import build
    build.build()


@pytest.mark.parametrize("name", sorted(HEADERS))
def test_exports_match_header(name):
    so = REPO / "n730_b200" / "lib" / name
    declared = _declared(HEADERS[name])
    assert declared, "no declarations parsed"
    missing = [s for s in declared if s not in _exported(so)]
    assert not missing, f"{name} lacks {missing}"


def test_reference_abi_complete():
    """All 26 symbols of the reference CUDA library and the 6 of its core are declared."""
    ref_cuda = """n730_cuda_init n730_cuda_destroy n730_load_activations n730_get_activations
    n730_upload_weight n730_upload_norm_weight n730_free_device_buf n730_rmsnorm n730_linear
    n730_residual_add n730_add_bias n730_swiglu n730_apply_rope n730_rope_precompute
    n730_softmax_scores n730_attention_forward n730_linear_from_buf n730_get_scores
    n730_attention_qk_only n730_device_alloc n730_device_free n730_memcpy_d2d n730_memcpy_h2d
    n730_memcpy_d2h n730_sync n730_cuda_version""".split()
    ref_core = "n730_open n730_close n730_read_layer n730_probe_layer_size n730_layer_elements n730_version".split()
    assert len(ref_cuda) == 26 and len(ref_core) == 6
    assert set(ref_cuda) <= set(_declared(HEADERS["n730_cuda.so"]))
    assert set(ref_core) <= set(_declared(HEADERS["n730core.so"]))


def test_ctypes_load_without_gpu():
    from n730_b200 import _lib
    lib = _lib.cuda()
    assert b"sm_100a" in lib.n730_cuda_version()
    assert _lib.core().n730_version()


def test_model_config_layout_matches_header():
    """The ctypes N730ModelConfig (n730_b200.engine) lists the header's fields in the same order
    and types: the struct crosses the C ABI by value layout."""
    import re

    from n730_b200.engine import N730ModelConfig
    hdr = (REPO / "include" / "n730_cuda.h").read_text()
    body = hdr[hdr.index("typedef struct N730ModelConfig {"):hdr.index("} N730ModelConfig;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for ctype, names in re.findall(r"\b(int32_t|float)\s+([^;]+);", body):
        fields += [(n.strip(), ctype) for n in names.split(",")]
    py = [(n, "float" if t.__name__ == "c_float" else "int32_t") for n, t in N730ModelConfig._fields_]
    assert py == fields
