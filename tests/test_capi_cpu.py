"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/qwen3_b200.h declares, rejects bad configs with the crate's error
kinds, and fails loudly (no CPU fallback) when no GPU is present."""
import ctypes
import json
import os
import re
import subprocess

import pytest

from oracle import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qwen3_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"QW_API\s+int\s+(qw_\w+)\s*\(", src)))


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_header_declares_entry_points():
    names = _declared()
    for n in ["qw_model_load", "qw_forward", "qw_generate_greedy", "qw_spec_generate", "qw_cache_truncate",
              "qw_kv_slice_update", "qw_quantized_matmul"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    import qwen3_b200 as q
    q.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", q.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(qw_\w+)$", out, flags=re.M))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    for n in _declared():
        assert hasattr(q.lib(), n)
        assert n in q.SIGNATURES, f"python mirror lacks {n}"


def test_version_and_last_error():
    import qwen3_b200 as q
    assert "sm_100a" in q.version()
    buf = ctypes.create_string_buffer(8)
    assert q.lib().qw_last_error(buf, 8) == 0


def test_config_errors_map_to_crate_errors():
    import qwen3_b200 as q
    with pytest.raises(q.InvalidConfig):
        q.Qwen3.init_random({"model_type": "qwen3"}, 1)
    with pytest.raises(q.InvalidConfig):
        q.lib()  # noqa
        h = ctypes.c_void_p()
        q.check(q.lib().qw_model_init_random(b"{not json", 1, 0, 0, 0, 1, ctypes.byref(h)))
    bad = dict(synth.tiny_config(), hidden_size=250, head_dim=None)
    with pytest.raises(q.InvalidConfig):
        q.Qwen3.init_random(bad, 1)


def test_model_load_missing_dir_is_model_load_error(tmp_path):
    import qwen3_b200 as q
    with pytest.raises(q.ModelLoad):
        q.Qwen3.load(str(tmp_path / "nope"))


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure mode")
def test_compute_without_gpu_fails_loudly():
    import qwen3_b200 as q
    with pytest.raises(q.CudaError):
        q.Qwen3.init_random(synth.tiny_config(), 1)
    with pytest.raises(q.Error):
        q.quantized_matmul(1, 1, 1, 1, 1, 1, 16, 64)


def test_unsupported_quantization_rejected():
    import qwen3_b200 as q
    cfg = dict(synth.tiny_config(), quantization=dict(group_size=32, bits=4))
    with pytest.raises((q.Unsupported, q.CudaError)):
        q.Qwen3.init_random(cfg, 1)
    cfg = dict(synth.tiny_config())
    cfg.pop("quantization")
    with pytest.raises((q.ModelLoad, q.CudaError)):
        q.Qwen3.init_random(cfg, 1)
    cfg = dict(synth.tiny_config(), model_type="gemma4")
    with pytest.raises(q.ModelLoad):
        q.Qwen3.init_random(cfg, 1)
    json.dumps(cfg)


def test_python_static_slot_count_matches_header():
    """qwen3_b200.STATIC_AMAX_SLOTS mirrors QW_STATIC_AMAX_SLOTS of the header."""
    import qwen3_b200 as q
    m = re.search(r"#define\s+QW_STATIC_AMAX_SLOTS\s+(\d+)", open(HEADER).read())
    assert m and int(m.group(1)) == q.STATIC_AMAX_SLOTS
