"""Place an unmodified copy of the reference (viragadel6/minimaxh3) under baseline/_ref.

    python baseline/install_reference.py --reference /path/to/minimaxh3

``pip install --target baseline/_ref <reference>`` does not work: the
reference has no setup.py or pyproject.toml.  This recipe stands in for it:
it copies every ``*.py`` file of the reference tree, byte for byte, into
``baseline/_ref`` (git-ignored; it travels with the working tree to a GPU
machine) and writes ``baseline/_ref/MANIFEST.sha256`` with each file's
SHA-256, so a reader can check that nothing was changed.  The benchmark's
same-box competitor imports ``kernels.fp8_attention`` / ``kernels.fp8_linear``
from there (the reference's own Triton kernels and wrappers).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of viragadel6/minimaxh3 (read only)")
    args = ap.parse_args(argv)
    src_root = os.path.abspath(args.reference)
    if not os.path.isfile(os.path.join(src_root, "kernels", "fp8_attention.py")):
        raise SystemExit(f"{src_root} does not look like the reference (kernels/fp8_attention.py missing)")
    if os.path.isdir(DEST):
        shutil.rmtree(DEST)
    lines = []
    for dirpath, _, files in sorted(os.walk(src_root)):
        for name in sorted(files):
            if not name.endswith(".py"):
                continue
            src = os.path.join(dirpath, name)
            rel = os.path.relpath(src, src_root)
            dst = os.path.join(DEST, rel)
            os.makedirs(os.path.dirname(dst), exist_ok=True)
            shutil.copyfile(src, dst)
            with open(dst, "rb") as f:
                lines.append(f"{hashlib.sha256(f.read()).hexdigest()}  {rel}")
    with open(os.path.join(DEST, "MANIFEST.sha256"), "w") as f:
        f.write("\n".join(lines) + "\n")
    print(f"copied {len(lines)} files to {DEST}")


if __name__ == "__main__":
    main()
