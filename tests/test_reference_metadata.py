"""The boundary accepts the reference's own LVSAMetadata
(lvsa/sparse_attention.py:286-353).  The reference object stores neither the
keyframe interval nor the offset; ``pattern_key`` reads the fields it does
store (geometry, W, expand_window, global_indices, rank, world), which fix
the pattern.  Here, on CPU: metadata built by the unmodified reference module
(skipped where the reference checkout is absent) gives, through that key,
the reference's own frame structures; and a duck-typed stand-in built from
the golden fixtures gives the same key as this package's metadata."""

import json
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest

from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

REF = os.environ.get("LVSA_REFERENCE_ROOT", "/root/reference")
PATS = np.load(os.path.join(GOLDEN, "patterns.npz"))
with open(os.path.join(GOLDEN, "patterns.json")) as fh:
    META = json.load(fh)


def standin(name):
    """A reference-shaped metadata object from the golden fixture (the fields
    the reference's LVSAMetadata carries and pattern_key reads)."""
    c = META[name]
    return SimpleNamespace(total_latent_frames=c["T"], num_patches=c["P"], window_size=c["W"],
                           n_first_frames=c["n_first"], key_frame_interval=c["kfi"],
                           expand_window=c["expand"], rank=c["rank"], world=c["world"],
                           global_indices=PATS[f"{name}.global_indices"].tolist(),
                           global_set=set(PATS[f"{name}.global_indices"].tolist()))


@pytest.mark.parametrize("name", sorted(META))
def test_pattern_key_reproduces_reference_structures(name):
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, pattern_key
    T, P, W, expand, gidx, rank, world = pattern_key(standin(name))
    # explicit globals, no anchors and no keyframe grid
    fp = O.frame_pattern(T, P, W, 0, None, 0, expand, rank, world, list(gidx))
    np.testing.assert_array_equal(fp["window_bounds"], PATS[f"{name}.window_bounds"])
    np.testing.assert_array_equal(fp["attended_indices"], PATS[f"{name}.attended_indices"])
    np.testing.assert_array_equal(fp["fi_indices"], PATS[f"{name}.fi_indices"])
    c = META[name]
    ours = LVSAMetadata.build(T, P, W, c["n_first"], c["kfi"], rank, world, expand_window=expand,
                              keyframe_offset=c["offset"], boundary_guards=c["guards"] or None)
    assert pattern_key(ours) == pattern_key(standin(name))


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "lvsa")), reason="reference checkout absent")
@pytest.mark.parametrize("args", [(9, 1560, 1, 1, 4, 0, 1, True, 3, None), (81, 1560, 2, 1, 4, 0, 1, True, 2, None),
                                  (21, 16, 3, 1, 5, 0, 1, False, 2, None), (20, 10, 2, 1, 5, 1, 2, True, 0, "guards")])
def test_reference_module_metadata_through_pattern_key(args):
    sys.path.insert(0, REF)
    from lvsa.sparse_attention import LVSAMetadata as RefMeta, compute_boundary_guard_frames
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, pattern_key
    T, P, W, nf, kfi, rank, world, expand, off, g = args
    guards = compute_boundary_guard_frames(T, T * P // world, P, world, W) if g else None
    ref = RefMeta.build(total_latent_frames=T, num_patches=P, window_size=W, n_first_frames=nf,
                        key_frame_interval=kfi, rank=rank, world=world, expand_window=expand,
                        keyframe_offset=off, boundary_guards=guards)
    key = pattern_key(ref)
    ours = LVSAMetadata.build(T, P, W, nf, kfi, rank, world, expand_window=expand, keyframe_offset=off,
                              boundary_guards=guards)
    assert key == pattern_key(ours)
    fp = O.frame_pattern(key[0], key[1], key[2], 0, None, 0, key[3], key[5], key[6], list(key[4]))
    np.testing.assert_array_equal(fp["window_bounds"], ref.window_bounds.numpy())
    np.testing.assert_array_equal(fp["attended_indices"], ref.attended_indices.numpy())
