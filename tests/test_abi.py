"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute: runs without a GPU)."""
import ctypes
import re
from pathlib import Path

import cmachine_b200 as cm

ROOT = Path(__file__).resolve().parent.parent


def declared(header: Path):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    text = re.sub(r"#.*", "", text)
    names = set()
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b([a-z_][a-z0-9_]*)\s*\(([^;{]*?)\)\s*;", text):
        prefix, name = m.group(1), m.group(2)
        if "typedef" in prefix or "(*" in m.group(0):
            continue
        names.add(name)
    return names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(cm.LIB_PATH))
    headers = ["gpu.h", "qwen.h", "qwen_b200.h"]
    missing = []
    total = 0
    for h in headers:
        for name in sorted(declared(ROOT / "include" / h)):
            total += 1
            if not hasattr(lib, name):
                missing.append(f"{h}:{name}")
    assert total > 80
    assert not missing, missing


def test_reference_primitive_names_are_all_present():
    """Every function of the reference's src/gpu.h (src/gpu.h:10-51) plus the
    three byte-cache entry points (src/qwen_cache.inc:13,20,35)."""
    names = """gpu_open gpu_close gpu_alloc gpu_free gpu_zero gpu_copy gpu_read gpu_write gpu_weight gpu_matvec
    gpu_rms gpu_rms_scale gpu_multiply gpu_plane gpu_plane_scaled gpu_linear2 gpu_identical_finite gpu_add
    gpu_bias gpu_rope gpu_cache gpu_attention gpu_swiglu gpu_gate_anchor gpu_gate_swiglu gpu_top2 gpu_sync
    gpu_weight_configure gpu_owned_weight gpu_owned_weight_bytes gpu_owned_embedding gpu_weight_release
    gpu_weight_info gpu_live_bytes gpu_peak_bytes gpu_free_bytes gpu_encode_current gpu_byte_attention
    gpu_ring_attention""".split()
    lib = ctypes.CDLL(str(cm.LIB_PATH))
    assert [n for n in names if not hasattr(lib, n)] == []


def test_python_mirror_declares_library():
    L = cm.lib()
    assert L.qwen_port_name(0) == b"input"
    assert L.qwen_port_name(13) == b"consumed_mlp_write"
    assert L.qwen_port_name(14) is None
