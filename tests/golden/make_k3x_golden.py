"""Write a K3X v1 container with the reference's own converter.

    python tests/golden/make_k3x_golden.py /path/to/reference

The reference's synthetic K3 checkpoint (reference/k3x_ref/fixtures.py,
write_source_checkpoint) with two experts per MoE layer, converted by
converter/k3x_converter/writer.py (convert) into tests/golden/k3x_small.k3x
(about 1 MB, mostly the 4 KB extent alignment): FP32 tensors, MXFP4 expert
records (UINT8 data + E8M0 auxiliary), layer and expert directories, CRC32C
and SHA-256 digests. The reference imports google_crc32c; the stand-in under
tests/golden/_shims is put on sys.path for that.
"""
from __future__ import annotations

import shutil
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path[:0] = [str(HERE / "_shims"), str(ref / "reference"), str(ref / "converter")]
    from k3x_converter.writer import convert
    from k3x_ref.config import SyntheticK3Config
    from k3x_ref.fixtures import write_source_checkpoint
    cfg = SyntheticK3Config.default().replace(num_experts=2, top_k=1)
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "source"
        write_source_checkpoint(src, config=cfg)
        out = Path(tmp) / "k3x_small.k3x"
        convert(src, out)
        shutil.copyfile(out, HERE / "k3x_small.k3x")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GLM5X_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: %s <reference project root> (or set GLM5X_REFERENCE_ROOT)" % sys.argv[0])
    main(root)
