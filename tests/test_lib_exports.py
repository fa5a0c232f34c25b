"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls: runs without a GPU)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "ornith-flight_b200", "libornith_cuda.so")
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", re.M)


def declared_functions():
    names = set()
    for h in ("gpu.h", "ornith_moe.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//.*", "", text)
        for m in DECL.finditer(text):
            name = m.group(1)
            if name not in ("if", "while", "sizeof", "defined"):
                names.add(name)
    return names


def test_headers_declare_the_boundary():
    names = declared_functions()
    for must in ("gpu_init", "gpu_alloc", "gpu_matmul", "gpu_expert_mlp", "gpu_router",
                 "gpu_topk_softmax", "gpu_moe_forward", "ofb_dequantize", "ofb_moe_forward",
                 "ofb_route"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_loads(ofb):
    assert ofb.lib.ofb_build_info().startswith(b"ornith-flight-b200")
    assert ofb.lib.ofb_status_string(1) == b"invalid argument"
