"""Generates tests/golden/philox_kat.json: cuRAND's Philox4x32-10 block
function evaluated on a B200 for a fixed list of (key, counter) inputs.

cuRAND is an independent implementation of the same published generator
(Salmon et al., SC'11) that crates/ops/src/rng.rs:43-60 implements, so its
outputs pin the oracle's restatement. Run on a GPU host:
    python tests/golden/make_philox_kat.py
"""
import json
import os
import random
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def cases():
    edge = [0, 1, 0x7FFFFFFF, 0x80000000, 0xFFFFFFFF]
    out = []
    for kk in [(0, 0), (0xFFFFFFFF, 0xFFFFFFFF), (0, 7), (0, 11), (1, 2)]:
        for c in [(0, 0, 0, 0), (1, 0, 0, 0), (0, 0, 1, 0), (10, 0, 3, 0),
                  (0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF)]:
            out.append((*kk, *c))
    rng = random.Random(2024)
    for _ in range(40):
        out.append(tuple(rng.choice(edge) if rng.random() < 0.2 else rng.getrandbits(32)
                         for _ in range(6)))
    return out


def main():
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "philox_curand")
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-o", exe,
                        os.path.join(HERE, "philox_curand.cu")], check=True)
        inp = "\n".join(" ".join(str(x) for x in c) for c in cases()) + "\n"
        res = subprocess.run([exe], input=inp, capture_output=True, text=True, check=True)
    lines = res.stdout.strip().splitlines()
    kat = {"generator": "cuRAND curand_Philox4x32_10 (CUDA 12.9) on sm_100a",
           "layout": "key = [key0, key1] (key0 = seed >> 32, key1 = seed & 0xffffffff); "
                     "ctr = [counter_lo, counter_hi, stream_lo, stream_hi]",
           "cases": []}
    for c, line in zip(cases(), lines):
        kat["cases"].append({"key": [c[0], c[1]], "ctr": list(c[2:]),
                             "out": [int(x) for x in line.split()]})
    with open(os.path.join(HERE, "philox_kat.json"), "w") as f:
        json.dump(kat, f, indent=1)
    print(f"wrote {len(kat['cases'])} cases")


if __name__ == "__main__":
    main()
