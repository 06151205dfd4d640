"""Places the unmodified reference (SwiftWare-Lab/lcd) under ``baseline/_ref`` so that its own
Numba-CUDA path can be timed on a GPU box, where the reference checkout does not exist.

The documented way - ``pip install --no-index --no-build-isolation --target baseline/_ref
<reference>`` - does not apply: the project has neither ``setup.py`` nor ``pyproject.toml`` (pip:
"not installable").  It is plain Python packages that are used by putting the checkout on
``PYTHONPATH``, so this script tries pip first and, when pip declines, mirrors the two packages the
hot path needs (``compiler/`` and ``utils/``: ``*.py`` files only) into ``baseline/_ref``.  That
directory is git-ignored: nothing of the reference enters this repository's history.

    python baseline/install_reference.py [<reference checkout>]
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
PACKAGES = ("compiler", "utils")


def install(reference="/root/reference", quiet=True):
    """Returns a one-line description of what was done (or why nothing was)."""
    if not os.path.isdir(os.path.join(reference, "compiler")):
        return f"no reference checkout at {reference}"
    pip = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                          "--find-links", "/opt/wheelhouse", "--target", TARGET, reference],
                         capture_output=True, text=True)
    if pip.returncode == 0:
        return "installed with pip"
    reason = (pip.stderr.strip().splitlines() or ["pip failed"])[-1]
    for package in PACKAGES:
        destination = os.path.join(TARGET, package)
        if os.path.isdir(destination):
            shutil.rmtree(destination)
        shutil.copytree(os.path.join(reference, package), destination,
                        ignore=lambda folder, names: [
                            name for name in names
                            if not (name.endswith(".py") or os.path.isdir(os.path.join(folder, name)))
                            or name in ("__pycache__", "fusion_benchmark", "transform_tests")])
    note = f"pip declined ({reason}); mirrored {', '.join(PACKAGES)} into baseline/_ref"
    if not quiet:
        print(note)
    return note


if __name__ == "__main__":
    print(install(*(sys.argv[1:2] or ["/root/reference"]), quiet=True))
