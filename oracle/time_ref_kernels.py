"""TEST INFRASTRUCTURE / MEASUREMENT ONLY — times the reference's own GPU
attention kernels on this machine's GPU beside this library's kernels.

The reference ships its GPU attention variants as bench programs
(gpu/fattn_{bench,wmma,wmma2,wmma3,sk,gqa,kplane,kvhalf}.cu), each with a
main() that times its kernels with CUDA events on gated causal prefill
chunks (f32 q, sigmoid gate, P = 256 or 512 query rows after a prefix of
pos_start cached rows). oracle/Makefile.ref compiles them unchanged for
sm_100a into oracle/_ref/bench_*; this script runs each at its built-in
shapes (and fattn_gqa also at the hd-128 shape) and then times
aspida_attn_prefill_gated - the drop-in for those kernels' swap point - on
the same shapes with seeded N(0, 0.3^2) inputs. It prints the reference
programs' own output followed by one JSON line of this library's times.

Usage (on a GPU box): python oracle/time_ref_kernels.py
"""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")

REF_RUNS = [
    ("bench_fattn_bench", []),        # k_fattn_attend_tile (hd 128, 32/8, P 256)
    ("bench_fattn_wmma", []),         # wmma tile kernel (hd 128, 32/8, P 256)
    ("bench_fattn_sk", ["8"]),        # split-K k_splitk + k_combine, S = 8 (hd 128, 32/8)
    ("bench_fattn_gqa", ["128", "32", "8", "256"]),   # k_fattn_tile_gqa at hd 128
    ("bench_fattn_gqa", []),          # hd 256, 16/2, P 256 (the hura dims)
    ("bench_fattn_wmma2", []),        # hd 256, 16/2, P 256
    ("bench_fattn_wmma3", []),        # hd 256, 16/2, P 512
    ("bench_fattn_kplane", []),       # hd 256, 16/2, P 512
    ("bench_fattn_kvhalf", []),       # hd 256, 16/2, P 512 (fp16 / Q8_0 caches)
]

OUR_SHAPES = ([(128, 32, 8, 256, ps) for ps in (0, 4096, 12288, 25344)] +
              [(256, 16, 2, 256, ps) for ps in (0, 4096, 12288, 25344)] +
              [(256, 16, 2, 512, ps) for ps in (12288, 25344, 37376)])


def run_reference():
    for name, args in REF_RUNS:
        path = os.path.join(REF, name)
        print(f"### {name} {' '.join(args)}", flush=True)
        if not os.path.exists(path):
            print("  (not built)", flush=True)
            continue
        try:
            r = subprocess.run([path] + args, capture_output=True, text=True, timeout=300)
            print(r.stdout.rstrip(), flush=True)
            if r.returncode:
                print(f"  (exit {r.returncode}) {r.stderr[-300:]}", flush=True)
        except subprocess.TimeoutExpired:
            print("  (timed out)", flush=True)


def run_ours():
    import torch
    sys.path.insert(0, ROOT)
    from aspida_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    st = torch.cuda.current_stream()
    res = []
    for hd, nq, nkv, P, ps in OUR_SHAPES:
        g = torch.Generator(device=dev).manual_seed(3)
        q = torch.randn(P, nq * hd, generator=g, device=dev) * 0.3
        gate = torch.randn(P, nq * hd, generator=g, device=dev) * 0.3
        K = (torch.randn(ps + P, nkv * hd, generator=g, device=dev) * 0.3).half()
        V = (torch.randn(ps + P, nkv * hd, generator=g, device=dev) * 0.3).half()
        out = torch.empty(P, nq * hd, device=dev)

        def call():
            rc = lib.aspida_attn_prefill_gated(q.data_ptr(), K.data_ptr(), V.data_ptr(),
                                               gate.data_ptr(), out.data_ptr(), nq, nkv, hd, P,
                                               ps, st.cuda_stream)
            if rc:
                raise RuntimeError(f"prefill_gated rc={rc}")

        for _ in range(5):
            call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(40):
            call()
        e1.record(st)
        torch.cuda.synchronize()
        res.append({"hd": hd, "nq": nq, "nkv": nkv, "P": P, "pos_start": ps,
                    "ms_per_chunk": round(e0.elapsed_time(e1) / 40, 4)})
    print(json.dumps({"ours": "aspida_attn_prefill_gated", "runs": res}), flush=True)


if __name__ == "__main__":
    run_reference()
    run_ours()
