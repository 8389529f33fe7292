"""Install the reference's own CPU golden of the attention path into baseline/_ref.

    python oracle/install_ref.py [/path/to/reference]

The reference's device kernels are SDAA C and cannot be built here, and
`pip install` of the reference needs torch_sdaa and the tecocc toolchain.  Its CPU
golden of the hot path is plain PyTorch:
``flash_attn_varlen_func`` in test/zoo/teco/flash_attention/flash_attention.py
(lines 79-140; fp32 matmul / softmax per sequence), imported by that file next to
test/zoo/teco/executor.py.  This recipe copies those two files, unmodified, into
baseline/_ref/zoo/ (git-ignored; it travels to the GPU box with the working tree)
and writes the one module they import that is not available here,
``prototxt_parser.prototxt_parser_main`` (only its ``parse`` name is imported; the
golden never calls it), as a stub.  bench.py --impl reference imports the golden
from there.  A manifest records the source paths and SHA-256 of the copied files.

The reshape_and_cache golden is a C++ Executor method
(test/zoo/teco/reshape_and_cache/reshape_and_cache.cpp:136-147) that does not
compile outside the reference's gtest/protobuf harness, so the reference arm uses
this repository's C restatement of it (oracle/reshape_and_cache.c) for that part.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
DEST = os.path.join(ROOT, "baseline", "_ref")
FILES = ("test/zoo/teco/executor.py", "test/zoo/teco/flash_attention/flash_attention.py")


def install(ref: str = "/root/reference") -> str:
    if not all(os.path.exists(os.path.join(ref, f)) for f in FILES):
        raise FileNotFoundError(f"reference golden sources not found under {ref}")
    zoo = os.path.join(DEST, "zoo")
    stub = os.path.join(DEST, "prototxt_parser")
    os.makedirs(zoo, exist_ok=True)
    os.makedirs(stub, exist_ok=True)
    manifest = {"source": ref, "files": {}}
    for f in FILES:
        src = os.path.join(ref, f)
        dst = os.path.join(zoo, os.path.basename(f))
        shutil.copyfile(src, dst)
        with open(src, "rb") as fh:
            manifest["files"][f] = hashlib.sha256(fh.read()).hexdigest()
    with open(os.path.join(stub, "__init__.py"), "w") as fh:
        fh.write("")
    with open(os.path.join(stub, "prototxt_parser_main.py"), "w") as fh:
        fh.write('"""Stand-in: the golden imports parse() for its prototxt harness only."""\n\n\n'
                 "def parse(*args, **kwargs):\n"
                 "    raise NotImplementedError('prototxt parsing is not part of the golden')\n")
    with open(os.path.join(DEST, "MANIFEST.json"), "w") as fh:
        json.dump(manifest, fh, indent=1)
    return DEST


def load_golden():
    """flash_attn_varlen_func of the installed reference golden (ImportError if the
    recipe has not run)."""
    zoo = os.path.join(DEST, "zoo")
    if not os.path.exists(os.path.join(zoo, "flash_attention.py")):
        raise ImportError("reference golden not installed: run oracle/install_ref.py")
    for p in (DEST, zoo):
        if p not in sys.path:
            sys.path.insert(0, p)
    import flash_attention  # noqa: E402  (the reference's module, unmodified)
    return flash_attention.flash_attn_varlen_func


if __name__ == "__main__":
    print(install(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
