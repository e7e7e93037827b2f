"""Loads the golden fixtures written by tests/golden/make_golden.py."""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

QUANT_CASES = ["cfg0_4bit", "cfg1_3bit", "cfg2_2bit_gqa", "ties_4bit", "nosink_4bit",
               "s2_4bit", "s1_4bit", "noout_3bit"]


def load_quant(name: str) -> dict:
    z = np.load(GOLDEN / f"quant_{name}.npz")
    d = {k: z[k] for k in z.files}
    B, S, C, G, bits, sink = (int(x) for x in d["meta"])
    d.update(B=B, S=S, C=C, G=G, bits=bits, sink=bool(sink), ratio=float(d["ratio"]),
             base=float(d["base"]))
    off = 1 if (d["sink"] and S > 1) else 0
    n = B * (S - off) * C
    for tag in ("k", "v"):
        if f"{tag}_mask" in d:
            d[f"{tag}_mask"] = np.unpackbits(d[f"{tag}_mask"])[:n].reshape(B, S - off, C).astype(bool)
    d["off"] = off
    return d


def load_misc() -> dict:
    z = np.load(GOLDEN / "misc.npz")
    return {k: z[k] for k in z.files}
