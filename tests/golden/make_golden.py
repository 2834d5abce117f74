"""Generate tests/golden/*.npz by running the reference's own fp32 kernels.

Needs a GPU and oracle/_ref/ref_harness (built from the reference sources by
oracle/Makefile.ref). Usage: python tests/golden/make_golden.py <out_dir>
"""
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")


def run(mode, payload, n_out):
    with tempfile.TemporaryDirectory() as d:
        fin, fout = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        with open(fin, "wb") as f:
            f.write(payload)
        subprocess.run([HARNESS, mode, fin, fout], check=True, timeout=120)
        out = np.fromfile(fout, dtype=np.float32)
    assert out.size == n_out
    return out


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    for c in cases.ATTN_CASES:
        Q, K, V, scale = cases.attn_inputs(c)
        hdr = struct.pack("<4if", c["nh"], c["nkv"], c["hd"], c["seq"], float(scale))
        o = run("attn", hdr + Q.tobytes() + K.tobytes() + V.tobytes(), c["nh"] * c["hd"])
        np.savez_compressed(os.path.join(out_dir, c["name"] + ".npz"), out=o)
        print("wrote", c["name"])
    for c in cases.ROPE_CASES:
        x, ff = cases.rope_inputs(c)
        hdr = struct.pack("<2if", c["dim"], c["pos"], c["base"])
        y = run("rope", hdr + x.tobytes() + ff.tobytes(), c["dim"])
        np.savez_compressed(os.path.join(out_dir, c["name"] + ".npz"), out=y)
        print("wrote", c["name"])
    for c in cases.CHUNK_CASES:
        q, g, K, V = cases.chunk_inputs(c)
        hdr = struct.pack("<5i", c["nq"], c["nkv"], c["hd"], c["P"], c["ps"])
        o = run("chunk", hdr + q.tobytes() + g.tobytes() + K.tobytes() + V.tobytes(),
                c["P"] * c["nq"] * c["hd"])
        np.savez_compressed(os.path.join(out_dir, c["name"] + ".npz"), out=o)
        print("wrote", c["name"])


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
