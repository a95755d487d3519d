"""Writes tests/golden/moe_small.npz: regression vectors of the CPU oracle
(oracle/moe_oracle.c) for one small MoE layer with a shared expert.

The reference stores no golden tensors for this path and MLX (whose
arithmetic defines it) cannot run here, so these vectors pin the oracle's own
restatement: any later change to the oracle or to the kernels that moves a
bit shows up against this file.  Inputs are stored with the outputs, so the
fixture does not depend on numpy's generators staying the same.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402

SHAPE = dict(H=128, E=8, k=2, I=64, Is=64)
T_PREFILL, T_DECODE = 24, 3
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "moe_small.npz")


def main():
    L = oracle.make_layer(seed=2024, **SHAPE)
    x = oracle.make_x(T_PREFILL, SHAPE["H"], seed=2024)
    out = {f"w_{n}": getattr(L, n) for n in
           ("wr", "gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b",
            "sgu_w", "sgu_s", "sgu_b", "sdn_w", "sdn_s", "sdn_b", "wg")}
    out["shape"] = np.array([SHAPE[c] for c in ("H", "E", "k", "I", "Is")], np.int32)
    out["x"] = x
    idx, sc, logits, probs = oracle.router(x, L.wr, SHAPE["k"])
    out.update(router_idx=idx, router_scores=sc, router_probs=probs, router_logits=logits)
    for mode in (0, 1, 3, 7):
        y, _, _, parts = oracle.moe_prefill(L, x, int8_mode=mode, parts=True)
        out[f"prefill_mode{mode}"] = y
        if mode == 3:   # the operands of the last bf16 add, for the tolerance
            out.update(mode3_routed=parts[0], mode3_shared=parts[1], mode3_termmax=parts[2])
    yd, _, _ = oracle.moe_decode(L, x[:T_DECODE])
    out["decode_y"] = yd
    ids = np.sort(np.random.default_rng(7).integers(0, SHAPE["E"], 32)).astype(np.int32)
    xg = oracle.make_x(32, SHAPE["H"], seed=7)
    out.update(gather_x=xg, gather_ids=ids,
               gather_int8_order0=oracle.gather_qmm_int8(xg, L.gu_w, L.gu_s, L.gu_b, ids, order=0),
               gather_int8_order1=oracle.gather_qmm_int8(xg, L.gu_w, L.gu_s, L.gu_b, ids, order=1))
    np.savez_compressed(OUT, **out)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
