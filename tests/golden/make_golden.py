"""Generate tests/golden/exl3_golden.npz from the REFERENCE's own compiled code.

Runs in the build container only (it needs oracle/_ref/libexl3ref.so, which
oracle/Makefile compiles from the read-only reference sources).  Everything in
the fixture is an output of the reference's src/exl3_codec.cpp or
src/exl3-ggml.cpp on the deterministic inputs of tests/golden/kat.py:

  cb_sha256[cb]                 SHA-256 of decode_codebook over all 65536 states
  inner_sha256[bits,cb]         SHA-256 of decode_inner(k=256, n=384) fp16 bits
  inner_head[bits,cb]           the first 2 rows of that matrix (768 values)
  recon_sha256[bits,cb]         SHA-256 of reconstruct() with the KAT scales
  mm_y_b{bits}_r{rows}          ggml_exl3_mul_mat output (4/6/8-bit mul1) or the
                                reference-codec loop (other bitrates), f32 input
  mm_y16_b{bits}_r1             same with the input rounded to fp16
  mm_cb{cb}_b4_r1               3inst / mcg codebooks through the loop, 4-bit
  rows_b{bits}_c{count}         ggml_exl3_get_rows output for the reference's ids
  h128_sha256 / h128_block5     hadamard128 over the probe blocks

Usage:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from oracle.oracle import Oracle, Reference  # noqa: E402
import kat  # noqa: E402

OUT = HERE / "exl3_golden.npz"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    ref = Reference()
    orc = Oracle()  # only for record packing, itself checked against the reference below
    k, n = kat.KAT_K, kat.KAT_N
    suh, svh = kat.kat_scales()
    data: dict[str, np.ndarray] = {}
    meta: dict[str, str] = {}
    for cb in range(3):
        meta[f"cb_sha256_{cb}"] = sha(ref.codebook_table(cb))
    for bits in range(1, 9):
        packed = kat.kat_packed(bits)
        meta[f"packed_sha256_{bits}"] = sha(packed)
        for cb in range(3):
            inner = ref.decode_inner(packed, k, n, bits, cb)
            meta[f"inner_sha256_{bits}_{cb}"] = sha(inner)
            data[f"inner_head_{bits}_{cb}"] = inner[:2].copy()
            meta[f"recon_sha256_{bits}_{cb}"] = sha(ref.reconstruct(packed, suh, svh, k, n, bits, cb))
        records = orc.pack_records(packed, suh, svh, k, n, bits)
        batches = (1, 4, 8) if bits in (4, 6, 8) else (1, 4)
        for rows in batches:
            x = kat.kat_input(rows)
            data[f"mm_y_b{bits}_r{rows}"] = ref.mul_mat(records, bits, k, n, x)
        x16 = kat.kat_input(1).astype(np.float16)
        data[f"mm_y16_b{bits}_r1"] = ref.mul_mat(records, bits, k, n, x16)
        if bits in (4, 6, 8):
            for count in (1, 3, 17):
                ids = kat.rows_ids(count, n)
                data[f"rows_b{bits}_c{count}"] = ref.get_rows(records, bits, k, n, ids)
    packed4 = kat.kat_packed(4)
    rec4 = orc.pack_records(packed4, suh, svh, k, n, 4)
    for cb in (0, 1):
        data[f"mm_cb{cb}_b4_r1"] = ref.mul_mat(rec4, 4, k, n, kat.kat_input(1), codebook=cb)
    h = ref.hadamard128(kat.kat_h128_blocks())
    meta["h128_sha256"] = sha(h)
    data["h128_block5"] = h[5].copy()
    data["meta_json"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays, {len(meta)} digests)")


if __name__ == "__main__":
    main()
