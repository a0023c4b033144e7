"""Install the reference's own kernel module for the same-box GPU comparison.

    python baseline/install_reference.py REFERENCE_DIR

The reference (goldbar123467/NVFP4-Group-Gemm) is a flat folder of single-file
submissions with no setup.py or pyproject.toml, so ``pip install --target
baseline/_ref REFERENCE_DIR`` refuses it ("not installable"). This script does what
that install would have done for a one-module project: it copies the active
submission, ``submission.py``, byte for byte into ``baseline/_ref/`` (git-ignored;
the copy's SHA-256 is checked against the source) and writes beside it the stub of
the harness module it imports (``from task import input_t, output_t``), which the
reference does not ship. Nothing in the module is changed; ``bench.py`` imports it
under the name ``nvfp4_reference_submission`` and calls its ``custom_kernel``.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
MODULE = "submission.py"
TASK_STUB = '''"""Stub of the evaluation harness's task module (not part of the reference).

The reference's submission imports only these two type names from it.
"""
input_t = tuple
output_t = list
'''


def _sha256(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def install(reference_dir: str) -> str:
    src = os.path.join(reference_dir, MODULE)
    if not os.path.isfile(src):
        raise SystemExit(f"{src} not found")
    os.makedirs(TARGET, exist_ok=True)
    dst = os.path.join(TARGET, MODULE)
    shutil.copyfile(src, dst)
    if _sha256(src) != _sha256(dst):
        raise SystemExit("copy differs from the source")
    with open(os.path.join(TARGET, "task.py"), "w") as f:
        f.write(TASK_STUB)
    with open(os.path.join(TARGET, "SOURCE_SHA256"), "w") as f:
        f.write(f"{_sha256(dst)}  {MODULE}\n")
    return dst


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    print(install(sys.argv[1]))
