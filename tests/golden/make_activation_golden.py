"""Write a GLM5XACT fixture with the reference's own writer.

    python tests/golden/make_activation_golden.py /path/to/reference

converter/glm5x_converter/activation.py:21-57 (write_bf16_activation) writes
tests/golden/activation_small.glm5xact: 5 tokens x 48 hidden BF16 values
(index % 29 - 14) * 0.01, the synthetic input pattern of the reference's GLM
expert bench (runtime/src/cuda_glm5x_real_expert_bench.cpp:421-425). The
reference imports google_crc32c; the stand-in under tests/golden/_shims is
put on sys.path for that.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def pattern(tokens: int, hidden: int):
    import torch
    idx = torch.arange(tokens * hidden, dtype=torch.int64)
    return ((idx % 29 - 14).to(torch.float32) * 0.01).reshape(tokens, hidden).to(torch.bfloat16)


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path[:0] = [str(HERE / "_shims"), str(ref / "converter")]
    from glm5x_converter.activation import write_bf16_activation
    write_bf16_activation(HERE / "activation_small.glm5xact", pattern(5, 48))


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GLM5X_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: %s <reference project root> (or set GLM5X_REFERENCE_ROOT)" % sys.argv[0])
    main(root)
