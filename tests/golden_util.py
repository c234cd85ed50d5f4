"""Loading of the golden fixtures made by tests/golden/make_golden.py."""
import glob
import json
import os

import numpy as np

from ugbsa.synth import input_digest, planted_inputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def names():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    rec = {k: z[k] for k in z.files}
    meta = json.loads(str(rec.pop("meta")))
    inp = meta["inp"]
    q, k, v, planted = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"],
                                      n_planted=inp["n_planted"], seed=inp["seed"],
                                      chained=inp["chained"], bf16=inp["bf16"])
    if input_digest(q, k, v) != str(rec["input_digest"]):
        raise AssertionError(f"{name}: regenerated inputs differ from the fixture's digest "
                             "(the synthetic generator changed)")
    return meta, (q, k, v), rec


CONFIGS = os.path.join(GOLDEN, "configs")


def load_config(name):
    """A BASELINE-configuration fixture (tests/golden/configs/, make_golden.py
    --configs): (meta, (q, k, v), record) with the inputs regenerated and checked."""
    z = np.load(os.path.join(CONFIGS, name + ".npz"))
    rec = {k: z[k] for k in z.files}
    meta = json.loads(str(rec.pop("meta")))
    inp = meta["inp"]
    q, k, v, _ = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"],
                                n_planted=inp["n_planted"], seed=inp["seed"],
                                chained=inp["chained"], bf16=inp["bf16"])
    if input_digest(q, k, v) != str(rec["input_digest"]):
        raise AssertionError(f"{name}: regenerated inputs differ from the fixture's digest")
    return meta, (q, k, v), rec


def unpack_sets(rec, S):
    """The fixture's canonical sets as a bool mask [B, H, Qt, NB]."""
    nb = (S + 63) // 64
    return np.unpackbits(rec["sets_ref"], axis=-1, count=nb).astype(bool)


def sets_mask(kv_idx, S):
    """Canonical sets of a kv_idx array (sentinel and causally invisible ids
    dropped) as a bool mask [B, H, Qt, NB]."""
    nb = (S + 63) // 64
    B, H, Qt, _ = kv_idx.shape
    last_blk = np.minimum(np.arange(Qt) * 64 + 63, S - 1) // 64
    ids = kv_idx.astype(np.int64)
    ok = (ids >= 0) & (ids < nb) & (ids <= last_blk[None, None, :, None])
    mask = np.zeros((B, H, Qt, nb), bool)
    b, h, t, j = np.nonzero(ok)
    mask[b, h, t, ids[b, h, t, j]] = True
    return mask


V1 = os.path.join(GOLDEN, "v1")


def v1_names():
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(V1, "*.npz")))


def load_v1(name):
    """A v1 per-row selector fixture (tests/golden/v1/, make_golden.py --v1):
    (meta, (q, k, v), record) with the inputs regenerated and checked, and the
    reference's keep mask unpacked to bool [B, H, S, NB] as record["keep"]."""
    z = np.load(os.path.join(V1, name + ".npz"))
    rec = {k: z[k] for k in z.files}
    meta = json.loads(str(rec.pop("meta")))
    inp = meta["inp"]
    q, k, v, _ = planted_inputs(inp["B"], inp["Hq"], inp["Hkv"], inp["S"], inp["D"],
                                n_planted=inp["n_planted"], seed=inp["seed"],
                                chained=inp["chained"], bf16=inp["bf16"])
    if input_digest(q, k, v) != str(rec["input_digest"]):
        raise AssertionError(f"{name}: regenerated inputs differ from the fixture's digest")
    rec["keep"] = np.unpackbits(rec["keep_ref"], axis=-1, count=int(rec["nb"])).astype(bool)
    return meta, (q, k, v), rec


def visible_mask(S):
    """[S, NB] bool: block j starts at or before row r."""
    nb = (S + 63) // 64
    return (np.arange(nb)[None, :] * 64) <= np.arange(S)[:, None]
