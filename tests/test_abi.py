"""The C-ABI library loads on a machine without a GPU and exports every
function include/clad3dgs_b200.h declares (no compute calls)."""

import ctypes
import re
from pathlib import Path

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
