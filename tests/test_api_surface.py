"""The Python package exports every function the tests call as sg.<name>(...)
(checked on CPU, without a GPU, so that a binding lost in an edit shows up in
the CPU suite rather than only on the GPU box)."""
import glob
import os
import re

import spindle_b200 as sg


def test_package_exports_what_the_tests_call():
    here = os.path.dirname(os.path.abspath(__file__))
    called = set()
    for path in glob.glob(os.path.join(here, "*.py")):
        called |= set(re.findall(r"\bsg\.([a-z_][a-z0-9_]*)\(", open(path).read()))
    missing = sorted(n for n in called if not hasattr(sg, n))
    assert not missing, missing
