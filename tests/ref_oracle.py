"""Access to the unmodified reference package (installed under baseline/_ref) as a test oracle."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def reference_available() -> bool:
    return os.path.isdir(os.path.join(REF, "dsv41_train"))


def import_reference():
    if REF not in sys.path:
        sys.path.append(REF)
    import dsv41_train  # noqa: F401

    return dsv41_train
