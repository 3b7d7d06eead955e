"""Generates the golden fixtures in this directory from the CPU oracle.

The reference ships no golden vectors for the sparse-conv path (its Python
conv_none.py / hashmap_fallback.py are absent and the WGSL port cannot run
here), so these fixtures pin the oracle restatement itself; the oracle is in
turn checked against brute force and dense F.conv3d by tests/test_oracle.py.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402
from oracle import sparse_conv_ref as R  # noqa: E402


def main():
    pkg = __graft_entry__.load_package()
    W = pkg.workloads
    cases = {}
    # C1 structure at reduced scale, rows shuffled, 16 channels
    w = W.make_workload(1, scale=0.3)
    perm = W.shuffle_rows(w.n, 1)
    coords = np.ascontiguousarray(w.coords[perm])
    rng = np.random.default_rng(11)
    f = rng.standard_normal((len(coords), 16)).astype(np.float32)
    wt = (rng.standard_normal((16, 3, 3, 3, 16)) / np.sqrt(27 * 16)).astype(np.float32)
    b = (0.1 * rng.standard_normal(16)).astype(np.float32)
    km = R.kmap_sorted(coords, w.spatial_shape)
    cases["subm_c1_small"] = dict(coords=coords, spatial_shape=np.array(w.spatial_shape), feats=f, weight=wt,
                                  bias=b, kmap=km, out=R.conv_gather(f, km, wt, b).astype(np.float32),
                                  kmap_dil2=R.kmap_sorted(coords, w.spatial_shape, dilation=2))
    # two batch entries sharing spatial coords
    c2 = np.concatenate([coords[:300], coords[:300]], 0)
    c2[300:, 0] = 1
    cases["subm_batch2"] = dict(coords=c2, kmap=R.kmap_sorted(c2, w.spatial_shape))
    # down / up on a C4-structured small shell union
    w4 = W.make_workload(4, scale=0.04)
    c4 = np.ascontiguousarray(w4.coords[W.shuffle_rows(w4.n, 4)])
    pc, dmap = R.down2_map(c4)
    umap = R.up2_map(c4, pc)
    f4 = rng.standard_normal((len(c4), 16)).astype(np.float32)
    wd = (rng.standard_normal((32, 2, 2, 2, 16)) / np.sqrt(8 * 16)).astype(np.float32)
    wu = (rng.standard_normal((16, 2, 2, 2, 32)) / np.sqrt(8 * 32)).astype(np.float32)
    gd = R.conv_gather(f4, dmap, wd).astype(np.float32)
    cases["downup_c4_small"] = dict(coords=c4, parent_coords=pc, dmap=dmap, umap=umap, feats=f4, w_down=wd,
                                    w_up=wu, out_down=gd, out_up=R.conv_gather(gd, umap, wu).astype(np.float32))
    for name, arrs in cases.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)
        print(name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
