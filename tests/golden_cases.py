"""Helpers that enumerate the golden fixture cases (tests only)."""
import hashlib

import numpy as np


def tree_prefixes(z):
    out = set()
    for k in z.files:
        if k.startswith(("cfg1_", "deep_")):
            a = k.index("_")
            out.add(k[: k.index("_", a + 1) + 1])
        else:
            out.add(k[: k.index("_") + 1])
    return sorted(out)


def regenerate_logits(z, prefix):
    """Full-size inputs are stored as seed + SHA-256; rebuild and verify them."""
    from ddtree_eagle3_patch_b200.synthetic import cfg1_logits, deep_logits
    if prefix + "logits" in z.files:
        return z[prefix + "logits"]
    if prefix.startswith("cfg1_"):
        x = cfg1_logits(seed=0)
    elif prefix.startswith("deep_"):
        x = deep_logits(seed=1, peak=16.0)
    else:
        raise KeyError(prefix)
    x = x.numpy()
    digest = hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()
    assert digest == str(z[prefix + "logits_sha256"]), "synthetic generator drifted from the fixture"
    return x


def same_up_to_value_ties(vals_a, ids_a, vals_b, ids_b):
    """Top-k rows agree except for the order of equal values."""
    if not np.array_equal(vals_a, vals_b):
        return False
    for ra, rb, va in zip(ids_a, ids_b, vals_a):
        for v in np.unique(va):
            sel = va == v
            if set(ra[sel].tolist()) != set(rb[sel].tolist()):
                # the last tie group may be cut at k: only require equal size
                if v != va.min():
                    return False
    return True
