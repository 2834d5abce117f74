"""Generate tests/golden/*.npz by running the reference's own fp32 kernels.

Needs a GPU and oracle/_ref/ref_harness + oracle/_ref/ref_q8 (built from the
reference sources by oracle/Makefile.ref).
Usage: python tests/golden/make_golden.py [<out_dir>] [--q8-only]
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
HARNESS_Q8 = os.path.join(ROOT, "oracle", "_ref", "ref_q8")


def run_raw(harness, mode, payload):
    with tempfile.TemporaryDirectory() as d:
        fin, fout = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        with open(fin, "wb") as f:
            f.write(payload)
        subprocess.run([harness, mode, fin, fout], check=True, timeout=120)
        with open(fout, "rb") as f:
            return f.read()


def run(mode, payload, n_out, harness=HARNESS):
    out = np.frombuffer(run_raw(harness, mode, payload), dtype=np.float32)
    assert out.size == n_out
    return out


def main_q8(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    for c in cases.Q8_QUANT_CASES:
        x = cases.q8_quant_inputs(c)
        raw = run_raw(HARNESS_Q8, "quant", struct.pack("<q", c["nblk"]) + x.tobytes())
        n = c["nblk"] * 32
        assert len(raw) == n + 2 * c["nblk"]
        q = np.frombuffer(raw[:n], dtype=np.int8)
        s = np.frombuffer(raw[n:], dtype=np.float16)
        np.savez_compressed(os.path.join(out_dir, c["name"] + ".npz"), q=q, scales=s)
        print("wrote", c["name"])
    for c in cases.Q8_GQA_CASES:
        q, g, K, V = cases.q8_gqa_inputs(c)
        hdr = struct.pack("<5i", c["nq"], c["nkv"], c["hd"], c["P"], c["ps"])
        o = run("gqa", hdr + q.tobytes() + g.tobytes() + K.tobytes() + V.tobytes(),
                c["P"] * c["nq"] * c["hd"], harness=HARNESS_Q8)
        np.savez_compressed(os.path.join(out_dir, c["name"] + ".npz"), out=o)
        print("wrote", c["name"])


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
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    out = args[0] if args else os.path.dirname(os.path.abspath(__file__))
    if "--q8-only" in sys.argv:
        main_q8(out)
    else:
        main(out)
        main_q8(out)
