"""Generate the reference-pinned parity fixtures -- TEST INFRASTRUCTURE ONLY.

Runs the reference trainer's own CUDA code (oracle/_ref/ref_harness_tiny, built
by `make -C oracle/ref_harness` from the reference sources) on seeded inputs
drawn with oracle/golden.py's generators, and stores its losses, LoRA
gradients and post-AdamW adapters as tests/golden/ref_tiny_*.npz.  Needs a GPU;
run once on the B200 box:

    python tests/golden/make_ref_fixtures.py --out tests/golden

The fixtures are committed; the CPU tests (tests/test_oracle.py) regenerate
the same inputs from the recorded seeds and check the golden against them.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle import golden as G  # noqa: E402
import ref_io  # noqa: E402

# (name, batch, seq, seed, token distribution)
CASES = [("b1s32", 1, 32, 101, "uniform"), ("b2s48", 2, 48, 202, "uniform"), ("b1s64zipf", 1, 64, 303, "zipf")]
ADAMW = (3e-4, 0.9, 0.999, 1e-8, 0.01)


def case_inputs(cfg, batch, seq, seed, dist):
    base = G.make_base_weights(cfg, seed)
    lora = G.make_lora(cfg, seed + 1)
    tok, tgt = G.make_tokens(cfg, batch, seq, seed + 2, dist=dist)
    return base, lora, tok, tgt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--harness", default=os.path.join(ROOT, "oracle", "_ref", "ref_harness_tiny"))
    a = ap.parse_args()
    cfg = G.CFG_TINY
    manifest = {}
    for name, batch, seq, seed, dist in CASES:
        base, lora, tok, tgt = case_inputs(cfg, batch, seq, seed, dist)
        with tempfile.TemporaryDirectory() as td:
            fin, fout = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
            ref_io.write_input(fin, cfg, base, lora, tok, tgt, ADAMW)
            r = subprocess.run([a.harness, "parity", fin, fout], capture_output=True, text=True, timeout=600)
            print(r.stdout.strip(), r.stderr.strip())
            r.check_returncode()
            losses, grads, after = ref_io.read_output(fout, cfg, batch)
        arrs = {"losses": losses}
        arrs.update({"grad/" + k: v for k, v in grads.items()})
        arrs.update({"after/" + k: v for k, v in after.items()})
        path = os.path.join(a.out, f"ref_tiny_{name}.npz")
        np.savez_compressed(path, **arrs)
        manifest[name] = {"batch": batch, "seq": seq, "seed": seed, "dist": dist, "adamw": ADAMW,
                          "losses": [float(x) for x in losses]}
        print("wrote", path)
    with open(os.path.join(a.out, "ref_tiny_manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)


if __name__ == "__main__":
    main()
