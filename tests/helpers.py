"""Test helpers: move oracle models into the engine's integer-artifact naming."""
import numpy as np

from oracle.exact_oracle import LIN_NAMES


def oracle_tensors(om):
    """{name: array} of an oracle model in the layout of include/exactb200.h."""
    t = {}
    group = om.layers[0]["q"].kind == "group"
    for i, L in enumerate(om.layers):
        t[f"L{i}.g1"], t[f"L{i}.g2"] = L["g1"], L["g2"]
        for nm in LIN_NAMES:
            lin = L[nm]
            t[f"L{i}.{nm}.w"] = lin.w
            t[f"L{i}.{nm}.M"] = lin.M.astype(np.int32) if group else lin.M.astype(np.int64)
            if lin.b is not None:
                t[f"L{i}.{nm}.b"] = lin.b
    t["gf"] = om.gf
    if hasattr(om, "emb_i8"):
        t["emb"] = om.emb_i8
        if not om.c["tie"]:
            t["head.w"] = om.head.w
    else:
        t["head.w"] = om.head.w
    t["head.M"] = om.head.M
    return t
