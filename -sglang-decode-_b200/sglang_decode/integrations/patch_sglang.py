"""Point an SGLang checkout's model runner at ScheduledTritonBackend (or back).

SGLang picks its attention backend class by import inside
``python/sglang/srt/model_executor/model_runner.py``.  Swapping that single import
line makes every Triton-backend model runner build ``ScheduledTritonBackend`` instead
(its unsupported cases fall back to the original Triton decode on their own).  Same
contract as the reference's ``scripts/patch_sglang.py``: the checkout must be the
pinned SGLang v0.4.6.post5 commit, the file must hold exactly one import site, and
nothing is written otherwise.

    python -m sglang_decode.integrations.patch_sglang /path/to/sglang [--revert]
"""
from __future__ import annotations

import argparse
import subprocess
from pathlib import Path

PINNED_COMMIT = "7e257cd666c0d639626487987ea8e590da1e9395"
RUNNER = Path("python/sglang/srt/model_executor/model_runner.py")
UPSTREAM_IMPORT = "from sglang.srt.layers.attention.triton_backend import TritonAttnBackend"
PATCHED_IMPORT = ("from sglang_decode.integrations.sglang_backend import "
                  "ScheduledTritonBackend as TritonAttnBackend")


class PatchError(RuntimeError):
    """The checkout is not the pinned commit or its import site is not unique."""


def checkout_commit(checkout: Path) -> str:
    try:
        return subprocess.check_output(["git", "-C", str(checkout), "rev-parse", "HEAD"], text=True,
                                       stderr=subprocess.DEVNULL).strip()
    except (OSError, subprocess.CalledProcessError) as exc:
        raise PatchError(f"{checkout} is not a git checkout of SGLang") from exc


def apply(checkout, revert=False, expected_commit=PINNED_COMMIT) -> Path:
    """Swap the import (or swap it back with ``revert``); returns the edited file.

    ``expected_commit=None`` skips the commit check (for copies that are not git
    checkouts); a drifting API is then the caller's responsibility.
    """
    checkout = Path(checkout)
    if expected_commit is not None:
        found = checkout_commit(checkout)
        if found != expected_commit:
            raise PatchError(f"expected SGLang commit {expected_commit}, found {found}; "
                             "a different commit may have a different backend API")
    path = checkout / RUNNER
    text = path.read_text()
    source, target = (PATCHED_IMPORT, UPSTREAM_IMPORT) if revert else (UPSTREAM_IMPORT, PATCHED_IMPORT)
    sites = text.count(source)
    if sites != 1:
        raise PatchError(f"{path}: expected exactly one import site, found {sites}; nothing changed")
    path.write_text(text.replace(source, target))
    return path


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("checkout", type=Path)
    parser.add_argument("--revert", action="store_true")
    args = parser.parse_args(argv)
    try:
        path = apply(args.checkout, args.revert)
    except PatchError as exc:
        raise SystemExit(str(exc)) from None
    print(f"updated {path}")


if __name__ == "__main__":
    main()
