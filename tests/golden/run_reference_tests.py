"""Run fni8-serve's own test suite on CPU with this repository's `fni8` package as its
kernels package — a drop-in check, run where the fni8-serve sources are available (pass
--reference, or set $FNI8_REFERENCE); the GPU box never runs it.

fni8-serve's package __init__ files import, at load time, two names from its kernels
package that lie outside the W8A8 path this repository provides: `fni8.quant.rotation`
(KV-cache rotation) and `fni8.Compressed` (the pipeline codec). They are stubbed here, in
this process only, with objects that raise NotImplementedError when used; everything else
the suite touches comes from this repository's `fni8`. The suite runs in place and writes
nothing into the checkout (no bytecode, no pytest cache). Its CUDA-only tests skip on a
host without a GPU.

    python tests/golden/run_reference_tests.py --reference <fni8-serve checkout> [pytest args]
"""
from __future__ import annotations

import argparse
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _install_out_of_scope_stubs() -> None:
    import fni8
    import fni8.quant

    def out_of_scope(*args, **kwargs):
        raise NotImplementedError("not part of the W8A8 drop-in")

    rotation = types.ModuleType("fni8.quant.rotation")
    rotation.rotate_last = out_of_scope
    rotation.hadamard_matrix = out_of_scope
    sys.modules["fni8.quant.rotation"] = rotation
    fni8.quant.rotation = rotation

    class Compressed:  # referenced at import time only
        def __init__(self, *args, **kwargs):
            out_of_scope()

    fni8.Compressed = Compressed


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=os.environ.get("FNI8_REFERENCE"),
                    help="fni8-serve checkout (default: $FNI8_REFERENCE)")
    a, pytest_args = ap.parse_known_args()
    if a.reference is None or not os.path.isdir(os.path.join(a.reference, "tests")):
        print("pass --reference <fni8-serve checkout> or set FNI8_REFERENCE", file=sys.stderr)
        return 2
    sys.dont_write_bytecode = True
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.path.insert(0, os.path.join(REPO, "fni8-serve_b200"))
    sys.path.insert(0, os.path.abspath(a.reference))
    _install_out_of_scope_stubs()
    import pytest

    os.chdir(a.reference)
    return pytest.main(["-p", "no:cacheprovider", "-q", "tests", *pytest_args])


if __name__ == "__main__":
    sys.exit(main())
