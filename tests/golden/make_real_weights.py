"""Cut the real-weight parity fixture from the reference's pinned Qwen3-0.6B tensors.

The reference ships two layer-0 weights of Qwen3-0.6B as raw bf16 files with
SHA-256 records (Strassen_MM_Focus/data/qwen3-0.6b-real-v001/tensors/
layer0_down_proj.{bf16,json}, layer0_q_proj.{bf16,json}; the fetch recipe is
Strassen_MM_Focus/tools/fetch_real_weights_v001.py).  The whole tensors are
10 MiB, so this script keeps two slices in the layout the GEMM consumes
(W^T, [in_features, out_features]):

* ``down_t``: down_proj^T rows 0:1024 (input features), columns 0:256 (output
  features) -- a [1024, 256] corner of the Qwen3-0.6B MLP down projection
  (the benchmark's config 2 down weight is down_proj^T);
* ``q_t``: q_proj^T, all 1024 input features, columns 0:256 -- query heads 0
  and 1 (head_dim 128), for the fused qk_norm_rope epilogue.

It checks each full tensor against the reference's SHA-256 record before
slicing and writes the slices as bf16 bit patterns plus their own SHA-256 to
``tests/golden/real_weights.npz`` / ``real_weights.json``.

Usage (in the build container, where the reference checkout exists):

    python tests/golden/make_real_weights.py --reference <path of the reference checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
DATA = Path("Strassen_MM_Focus/data/qwen3-0.6b-real-v001/tensors")

SLICES = {
    # name: (tensor file stem, rows of W^T, columns of W^T)
    "down_t": ("layer0_down_proj", (0, 1024), (0, 256)),
    "q_t": ("layer0_q_proj", (0, 1024), (0, 256)),
}


def slice_sha256(bits: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits).astype("<u2").tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    arrays, records = {}, {}
    for name, (stem, rows, cols) in SLICES.items():
        meta = json.loads((args.reference / DATA / f"{stem}.json").read_text())
        raw = (args.reference / DATA / f"{stem}.bf16").read_bytes()
        digest = hashlib.sha256(raw).hexdigest()
        if digest != meta["sha256"] or len(raw) != meta["bytes"]:
            raise SystemExit(f"{stem}: SHA-256 {digest} does not match the reference's record")
        out_f, in_f = meta["shape"]  # [output_features, input_features]
        w = np.frombuffer(raw, dtype="<u2").reshape(out_f, in_f)
        wt = w.T[rows[0]:rows[1], cols[0]:cols[1]].copy()
        arrays[name] = wt
        records[name] = {"tensor": meta["name"], "tensor_sha256": meta["sha256"], "tensor_shape": meta["shape"],
                         "transposed_rows": list(rows), "transposed_cols": list(cols),
                         "slice_shape": list(wt.shape), "slice_sha256": slice_sha256(wt)}
    np.savez_compressed(HERE / "real_weights.npz", **arrays)
    (HERE / "real_weights.json").write_text(json.dumps(records, indent=1) + "\n")
    print(json.dumps(records, indent=1))


if __name__ == "__main__":
    main()
