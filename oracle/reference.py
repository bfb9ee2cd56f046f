"""Locates and imports the reference (sjjeong94/asrback, pure Python/PyTorch)
for the checkers. Test infrastructure: only the tests, the fixture script
(``tests/golden/make_golden.py``) and ``bench.py``'s CPU-baseline legs use it;
the product path never does.

Where the reference is looked for, in order:

1. ``$ASRBACK_REFERENCE``: a checkout (``<dir>/src/asrback``) or a directory
   holding the ``asrback`` package itself;
2. ``baseline/_ref`` of this repository (git-ignored), where
   ``python -m oracle.reference --install <checkout>`` lays the package down.

``pip install --target baseline/_ref <checkout>`` is the usual route, but the
checkout builds with hatchling, which this image does not have, so the install
copies the package's source files (``src/asrback/**/*.py``) as a wheel would
place them. Nothing under ``baseline/_ref`` is committed.

The reference imports ``asrfront`` (its audio front end, ``asrfront==0.2.2``
on PyPI), which is not installed; none of the code the checkers run calls
into it, so a stub module with the constants read at import time stands in.
"""

from __future__ import annotations

import argparse
import os
import shutil
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
INSTALL_DIR = REPO / "baseline" / "_ref"

__all__ = ["find", "load", "install", "install_asrfront_stub", "INSTALL_DIR"]


def install_asrfront_stub() -> None:
    """An ``asrfront`` with the module constants the reference reads at import."""
    if "asrfront" in sys.modules:
        return
    constants = dict(SAMPLE_RATE=16000, N_SAMPLES=480000, HOP_LENGTH=160, MAX_SAMPLES=480000,
                     N_MELS=128)
    stub = types.ModuleType("asrfront")
    for name in ("whisper", "qwen3_asr", "sensevoice", "gemma4"):
        setattr(stub, name, types.SimpleNamespace(**constants))

    def unavailable(*args, **kwargs):
        raise RuntimeError("asrfront is not installed (stub)")

    stub.load = unavailable
    for name in ("whisper", "qwen3_asr", "sensevoice", "gemma4"):
        getattr(stub, name).log_mel = unavailable
    sys.modules["asrfront"] = stub


def _package_parent(path: Path) -> Path | None:
    """The directory that holds ``asrback/__init__.py`` under ``path``."""
    for candidate in (path / "src", path):
        if (candidate / "asrback" / "__init__.py").is_file():
            return candidate
    return None


def find() -> Path | None:
    """The directory to put on ``sys.path`` for ``import asrback``, or None."""
    given = os.environ.get("ASRBACK_REFERENCE")
    if given:
        found = _package_parent(Path(given))
        if found is not None:
            return found
    return _package_parent(INSTALL_DIR)


def load() -> types.SimpleNamespace:
    """Imports the reference's ``whisper``, ``qwen3_asr`` and ``transcription``
    modules (raises ``ImportError`` when the reference is not found)."""
    root = find()
    if root is None:
        raise ImportError("the asrback reference was not found ($ASRBACK_REFERENCE or "
                          f"{INSTALL_DIR})")
    install_asrfront_stub()
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    from asrback import transcription
    from asrback.models import qwen3_asr, whisper

    return types.SimpleNamespace(whisper=whisper, qwen3_asr=qwen3_asr,
                                 transcription=transcription, root=root)


def install(checkout: Path, dest: Path = INSTALL_DIR) -> Path:
    """Copies the ``asrback`` package of ``checkout`` to ``dest/asrback``."""
    source = _package_parent(Path(checkout))
    if source is None:
        raise FileNotFoundError(f"no asrback package under {checkout}")
    target = Path(dest) / "asrback"
    if target.exists():
        shutil.rmtree(target)
    shutil.copytree(source / "asrback", target,
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    return target


def main() -> None:
    parser = argparse.ArgumentParser(description="install or locate the asrback reference")
    parser.add_argument("--install", metavar="CHECKOUT", default=None,
                        help="copy CHECKOUT's asrback package into baseline/_ref")
    args = parser.parse_args()
    if args.install:
        print(install(Path(args.install)))
    print(find())


if __name__ == "__main__":
    main()
