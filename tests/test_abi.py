"""The C-ABI library loads on a machine without a GPU and exports every
function include/clad3dgs_b200.h declares (no compute calls)."""

import ctypes
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, re.M):
            name = m.group(1)
            if name not in {"if", "while", "for", "return", "sizeof"}:
                names.add(name)
    return names


def test_header_declares_the_reference_symbols():
    names = declared_functions()
    for symbol in ("sh_consumer_sgd", "sh_consumer_adam", "sh_consumer_split_adam",
                   "sh_consumer_split_torch_adam", "launch_activation_consume",
                   "launch_quaternion_backward"):
        assert symbol in names


def test_library_exports_every_declared_symbol():
    import _native

    lib = ctypes.CDLL(str(_native.LIBRARY))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    import _native

    assert set(_native.exported_symbols()) == declared_functions()
    _native.library()  # argtypes bind without a GPU


def test_product_modules_do_not_reach_the_oracle():
    """The product path never imports or loads anything under oracle/."""
    for path in (ROOT / "clad-3dgs_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "oracle/" not in text, path
        assert "torch_cpu_path" not in text, path


@pytest.mark.parametrize("mirror,c_name", [("ShardUpdateArgs", "clad3dgs_shard_update_args"),
                                            ("AdamConfig", "AdamConfig"),
                                            ("TorchAdamConfig", "TorchAdamConfig")])
def test_struct_layouts_match_header(tmp_path, mirror, c_name):
    """Each ctypes mirror of a header struct has the C struct's size and
    every field at the C offset (a probe compiled with gcc against
    include/clad3dgs_b200.h)."""
    import _native
    from torch.utils.cpp_extension import CUDA_HOME

    if shutil.which("gcc") is None or CUDA_HOME is None:
        pytest.skip("gcc or the CUDA headers are not available")
    struct = getattr(_native, mirror)
    fields = [name for name, _ in struct._fields_]
    probe = tmp_path / "probe.c"
    probe.write_text(
        "#include <stdio.h>\n#include <stddef.h>\n#include \"clad3dgs_b200.h\"\n"
        "int main(void) {\n"
        f"  printf(\"size %zu\\n\", sizeof({c_name}));\n"
        + "".join(f"  printf(\"{f} %zu\\n\", offsetof({c_name}, {f}));\n"
                  for f in fields)
        + "  return 0;\n}\n")
    exe = tmp_path / "probe"
    cuda_include = os.path.join(CUDA_HOME, "include")
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", f"-I{cuda_include}",
                    str(probe), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run(
        [str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(struct)
    for f in fields:
        assert int(out[f]) == getattr(struct, f).offset, f


def _declared_arity():
    """Parameter count of every function the header declares."""
    arity = {}
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\(([^;{]*?)\)\s*;", text, re.S):
            name, params = m.group(1), m.group(2).strip()
            if name in {"if", "while", "for", "return", "sizeof"}:
                continue
            depth, count = 0, 0 if params in ("", "void") else 1
            for ch in params:
                depth += ch == "("
                depth -= ch == ")"
                count += ch == "," and depth == 0
            arity[name] = count
    return arity


def test_binding_argument_counts_match_header():
    """Every ctypes signature takes as many arguments as the header's
    prototype declares."""
    import _native

    arity = _declared_arity()
    signatures = _native._SIGNATURES
    assert set(signatures) <= set(arity)
    wrong = {name: (len(argtypes), arity[name]) for name, (_, argtypes) in signatures.items()
             if len(argtypes) != arity[name]}
    assert not wrong, wrong
