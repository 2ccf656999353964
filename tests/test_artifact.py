"""Exact release artifact: float64 conversion against the reference's converters, write/load round
trip with SHA-256 verification, and (GPU) a model loaded from a release against the reference's
logits."""
import json
import os

import numpy as np
import pytest

from oracle import exact_oracle as eo
from oracle import synth
from tests.helpers import oracle_tensors


def _convert_golden(golden):
    g = golden["convert"]
    c = dict(g["config"])
    return g, c, synth.float_checkpoint(c, g["seed"])


def test_conversion_matches_reference(golden):
    """Per-channel (qlin_chunked) and group-128 (GQLin) float64 conversion give the reference's
    integers bit for bit."""
    from exact_llm_b200 import artifact
    g, c, f = _convert_golden(golden)
    for nm, want in g["mats"].items():
        w, b = f[nm + ".weight"], f.get(nm + ".bias")
        qw, qM, qb = artifact.quantize_channel(w, b, chunk=100)
        assert eo.h16(qw) == want["ch_w"] and eo.h16(qM) == want["ch_M"]
        assert (qb is None and want["b"] is None) or eo.h16(qb) == want["b"]
        gw, gM, _ = artifact.quantize_group(w, b)
        assert eo.h16(gw) == want["g_w"] and eo.h16(gM) == want["g_M"]
    t = artifact.convert_checkpoint(f.__getitem__, c, lin="channel")
    assert eo.h16(t["emb_q16"]) == g["emb_q16"]


def test_release_round_trip_and_tamper(golden, tmp_path):
    """write_artifact -> load_artifact returns every tensor and the shipped tables unchanged; a
    single changed byte in any file is refused by its SHA-256."""
    from exact_llm_b200 import artifact, tables
    g, c, f = _convert_golden(golden)
    t = artifact.convert_checkpoint(f.__getitem__, c, lin="group")
    man = artifact.write_artifact(str(tmp_path), c, t, rope_len=64, lin="group")
    assert man["spec"] == artifact.SPEC and man["format"] == "Q16"
    arch, t2, tabs = artifact.load_artifact(str(tmp_path))
    assert arch["NL"] == c["NL"] and arch["lin"] == "group" and arch["rope_len"] == 64
    assert set(t2) == set(t)
    for k in t:
        assert np.array_equal(np.asarray(t2[k]), t[k]), k
    assert np.array_equal(np.asarray(tabs["exp"]), tables.exp_table())
    cos, _ = tables.rope_tables(64, c["hd"], c["theta"])
    assert np.array_equal(np.asarray(tabs["cos"]), cos[:, :c["hd"] // 2])
    with open(os.path.join(tmp_path, "manifest.json")) as fh:
        assert json.load(fh)["files"]["weights.int8"]["sha256"] == man["files"]["weights.int8"]["sha256"]
    del t2, tabs
    for fn in artifact.FILES:
        p = os.path.join(tmp_path, fn)
        with open(p, "r+b") as fh:
            fh.seek(17)
            b = fh.read(1)
            fh.seek(17)
            fh.write(bytes([b[0] ^ 1]))
        with pytest.raises(ValueError, match="SHA-256"):
            artifact.load_artifact(str(tmp_path))
        with open(p, "r+b") as fh:
            fh.seek(17)
            fh.write(b)
    artifact.load_artifact(str(tmp_path))


@pytest.mark.gpu
def test_release_models_run_on_gpu(golden, cuda_ok, tmp_path):
    """A release converted from float64 weights (per channel) reproduces the logits of the
    reference's own IntModel on those weights; a group-128 release of the synthetic tiny model
    reproduces its reference prefill."""
    from exact_llm_b200 import ExactModel, artifact
    g, c, f = _convert_golden(golden)
    t = artifact.convert_checkpoint(f.__getitem__, c, lin="channel")
    artifact.write_artifact(str(tmp_path / "ch"), c, t, rope_len=64, lin="channel")
    m = ExactModel.from_artifact(str(tmp_path / "ch"), max_batch=1)
    assert eo.h16(m(g["ids"])) == g["logits"]
    m.close()
    gm = golden["models"]["tiny-g128"]
    om = synth.build_model(dict(gm["config"]), gm["seed"])
    artifact.write_artifact(str(tmp_path / "g"), om.c, oracle_tensors(om), rope_len=64, lin="group")
    m = ExactModel.from_artifact(str(tmp_path / "g"), max_batch=1)
    assert eo.h16(m(gm["prompt"])) == gm["prefill"]
