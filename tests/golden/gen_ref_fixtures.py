"""Generates tests/golden/ref_*.npz: outputs of the REFERENCE's own SageAttention2
kernels (platform/spl-nn/cuda/sage_{common,quant,attn}.cu, built from the
reference sources into oracle/_ref by oracle/Makefile) on small seeded inputs.

Run on a machine with a B200 and oracle/_ref built:
    python tests/golden/gen_ref_fixtures.py
The inputs are not stored: they are regenerated bit-exactly from the seed by
the SplitMix64 generator of platform/spl-nn/src/sage/tests.rs:300-329
(oracle/sage_oracle.c:or_synthetic); a hash of them is stored to detect drift.
tests/test_golden.py then checks the CPU oracle against these files without a
GPU, which pins the oracle to the reference implementation."""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

CASES = {
    "dense": dict(),
    "nosmooth": dict(smooth=False),
    "merge2": dict(merge=2),
    "merge4": dict(merge=4),
    "pv16": dict(pv16=True),
}


def input_hash(x) -> str:
    h = hashlib.sha256()
    for a in (x.q, x.k, x.v):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    import sagetest as st
    from oracle import oracle as O
    for d in (64, 128):
        for name, kw in CASES.items():
            lay = st.small_layout()
            c = st.Case(batch=1, heads=2, kv_heads=2, tokens=lay.frames * lay.tokens_per_frame(), d=d, layout=lay,
                        seed=17 + d, **kw)
            x = st.make_inputs(c)
            out, q = st.run_reference_gpu(c, x)
            path = os.path.join(HERE, f"ref_d{d}_{name}.npz")
            np.savez_compressed(path, q8=q.q8, q_scale=q.q_scale, k8=q.k8, k_scale=q.k_scale, v8=q.v8,
                                stats=q.stats, kbias=q.kbias, out=out.astype(np.float32),
                                input_sha256=np.array(input_hash(x)),
                                meta=np.array([c.batch, c.heads, c.tokens, d, c.merge, int(c.smooth), int(c.pv16),
                                               c.seed], np.int64))
            print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
