"""Write packed expert sidecars with the reference's own cache writer.

    python tests/golden/make_sidecar_golden.py /path/to/reference

GLM5XPackedExpertCache.put (reference/glm5x_ref/packed_cache.py:327-404) on
two seeded small experts (gate/up [128, 64], down [64, 128], weights
N(0, 0.02) in BF16 from torch.Generator seed 2026):

- nvfp4: the weights packed by the reference's quantize_nvfp4_weight
  (nvfp4.py:180-198, scale_mode "mse"), stored as layer 10 expert 3 ->
  tests/golden/sidecar/layer-0010-expert-0003.pn4;
- mxfp4: the BF16 weights, encoded by put itself with encode_mxfp4
  (group 32, max_abs), stored as layer 10 expert 4 ->
  tests/golden/sidecar/layer-0010-expert-0004.pm4.

tests/golden/sidecar/expected.json records, per role, what the reference's
own reader returns for each file (GLM5XPackedExpertCache._decode_role,
packed_cache.py:407-504, run on the CPU): the SHA-256 of the NVFP4 packed
bytes, of the blocked E4M3 scale bytes and the FP32 global scale; for MXFP4
the SHA-256 of the BF16 weights it decodes (decode_mxfp4, mxfp4.py:110-144).
The reference imports google_crc32c; the stand-in under tests/golden/_shims
is put on sys.path for that.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import struct
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "sidecar"
DIGEST = "glm5x-b200-sidecar-fixture-0001"


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path[:0] = [str(HERE / "_shims"), str(ref / "reference"), str(ref / "converter")]
    import torch
    from glm5x_ref.layer10_moe import GLM5XExpertWeights
    from glm5x_ref.nvfp4 import quantize_nvfp4_weight
    from glm5x_ref.packed_cache import GLM5XPackedExpertCache

    g = torch.Generator().manual_seed(2026)
    I, H = 128, 64
    bf16 = [(torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16)
            for shape in ((I, H), (I, H), (H, I))]
    OUT.mkdir(exist_ok=True)
    expected = {"source_digest": DIGEST, "files": {}}
    with tempfile.TemporaryDirectory() as tmp:
        cache = GLM5XPackedExpertCache(tmp)
        nv = GLM5XExpertWeights(*[quantize_nvfp4_weight(w, scale_mode="mse") for w in bf16])
        cache.put((10, 3), DIGEST, nv, precision="nvfp4")
        cache.put((10, 4), DIGEST, GLM5XExpertWeights(*bf16), precision="mxfp4")
        for key, precision, suffix in (((10, 3), "nvfp4", "pn4"), ((10, 4), "mxfp4", "pm4")):
            name = f"layer-{key[0]:04d}-expert-{key[1]:04d}.{suffix}"
            data = (Path(tmp) / name).read_bytes()
            shutil.copyfile(Path(tmp) / name, OUT / name)
            (magic, version, mlen) = struct.unpack_from("<8sII", data)
            meta = json.loads(data[16:16 + mlen])
            payload = data[16 + mlen:]
            roles = []
            for role in meta["roles"]:
                dec = GLM5XPackedExpertCache._decode_role(role, payload, device=torch.device("cpu"),
                                                          precision=precision)
                if precision == "nvfp4":
                    roles.append({
                        "shape": list(dec.shape),
                        "packed_sha256": hashlib.sha256(dec.packed.numpy().tobytes()).hexdigest(),
                        "scales_sha256": hashlib.sha256(
                            dec.scales.view(torch.uint8).numpy().tobytes()).hexdigest(),
                        "global_scale": float(dec.global_scale.item()),
                    })
                else:
                    roles.append({
                        "shape": list(dec.shape),
                        "decoded_bf16_sha256": hashlib.sha256(
                            dec.view(torch.int16).numpy().tobytes()).hexdigest(),
                    })
            expected["files"][name] = {"precision": precision, "roles": roles}
    (OUT / "expected.json").write_text(json.dumps(expected, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GLM5X_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: %s <reference project root> (or set GLM5X_REFERENCE_ROOT)" % sys.argv[0])
    main(root)
