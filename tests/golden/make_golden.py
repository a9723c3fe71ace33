"""Generate tests/golden/golden_v1.json from the reference's binary64 scalar oracle.

Runs Rosevine's own independent reference math, scripts/correctness_oracle.py (imported from a
Rosevine checkout given by --reference), and its scalar operator
fixture research/fixtures/scalar-operators-v1.json, on seeded inputs, and writes the results as
a small JSON fixture. The committed fixture is what the tests read; the reference checkout is
only needed to regenerate it:

    python tests/golden/make_golden.py --reference /path/to/Rosevine
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import random
import struct

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    spec = importlib.util.spec_from_file_location("correctness_oracle",
                                                  os.path.join(root, "scripts", "correctness_oracle.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with open(os.path.join(root, "research", "fixtures", "scalar-operators-v1.json")) as f:
        fixture = json.load(f)
    return mod, fixture


def f16_bytes(v: float) -> bytes:
    return struct.pack("<e", v)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a Rosevine checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_v1.json"))
    args = ap.parse_args()
    C, fixture = load_reference(args.reference)
    rnd = random.Random(20261201)
    g: dict = {"source": "scripts/correctness_oracle.py (binary64) and research/fixtures/scalar-operators-v1.json",
               "generator": "tests/golden/make_golden.py"}

    # Q4_0 block decode, including the all-nibbles pattern of test_correctness_oracle.py.
    blocks = []
    patterns = [bytes((15 - i) * 16 + i for i in range(16)), bytes(range(0, 256, 16)), bytes(16),
                bytes([0xff] * 16)] + [bytes(rnd.randrange(256) for _ in range(16)) for _ in range(4)]
    for scale in [0.0, 1.0, -2.0, 2 ** -24, 0.0137, 65504.0]:
        for p in patterns:
            blk = f16_bytes(scale) + p
            blocks.append({"block": blk.hex(), "values": C.q4_0_decode(blk)})
    g["q4_0_decode"] = blocks

    # tanh GELU (binary64) on the fixture's inputs plus a grid; criterion from the fixture.
    xs = list(fixture["gelu_tanh"]["input"]) + [i / 16 for i in range(-96, 97)]
    g["gelu_tanh"] = {"input": xs, "output": C.gelu_tanh(xs), "criterion": fixture["criterion"]}

    # Softmax of the fixture's extreme logits (binary64).
    sm = fixture["softmax"]["input"]
    g["softmax"] = {"input": sm, "output": C.softmax(sm)}

    # Router selection weights: the reference's known answer plus seeded 128-expert rows whose
    # top-9 are separated by > 1e-3 (no near ties), ids taken from the binary64 ranking.
    cases = [{"logits": [0.0, math.log(3), 0.0], "ids": [1, 0]}]
    while len(cases) < 12:
        lg = [rnd.gauss(0.0, 1.06) for _ in range(128)]
        rank = sorted(range(128), key=lambda i: (-lg[i], i))
        if min(lg[rank[j]] - lg[rank[j + 1]] for j in range(8)) > 1e-3:
            cases.append({"logits": lg, "ids": rank[:8]})
    for c in cases:
        r = C.router_selected_weights(c["logits"], c["ids"])
        c["weights"] = r["weights"]
        c["probabilities"] = r["probabilities"]
    g["router_selected_weights"] = cases
    g["router_underflow"] = {"logits": [0.0, -1000.0], "ids": [1],
                             "weights": C.router_selected_weights([0.0, -1000.0], [1])["weights"],
                             "denominator": C.router_selected_weights([0.0, -1000.0], [1])["normalization_denominator"]}

    # Gated FFN fixture (GELU on gate, times up, then down), binary64.
    gf = fixture["gated_ffn"]
    g["gated_ffn"] = {"fixture": gf,
                      "result": C.gated_ffn(gf["input"], gf["up_matrix_rows"], gf["gate_matrix_rows"],
                                            gf["down_matrix_rows"])}

    # Q4_0 x Q8_0 rows: exact binary64 dot of the decoded operands, for k in {32, 96, 704, 2816}.
    dots = []
    for k in [32, 96, 704, 2816]:
        for it in range(3):
            row = b""
            xq = b""
            for b in range(k // 32):
                row += f16_bytes(rnd.choice([0.01, -0.1, 3.0, 6e-8, 0.0137])) + bytes(rnd.randrange(256) for _ in range(16))
                q = [rnd.randrange(-127, 128) for _ in range(32)]
                if it == 2:  # extreme quants: every weight -8, every activation -127 or +127
                    row = row[:-16] + bytes(16)
                    q = [127 if (b % 2) else -127] * 32
                xq += f16_bytes(rnd.choice([0.004, 0.03, 1.5])) + struct.pack("<32b", *q)
            wv, xv = [], []
            for b in range(k // 32):
                wv += C.q4_0_decode(row[18 * b:18 * b + 18])
                d = struct.unpack("<e", xq[34 * b:34 * b + 2])[0]
                xv += [d * v for v in struct.unpack("<32b", xq[34 * b + 2:34 * b + 34])]
            exact = math.fsum(a * c for a, c in zip(wv, xv))
            magnitude = math.fsum(abs(a * c) for a, c in zip(wv, xv))
            dots.append({"k": k, "row": row.hex(), "xq": xq.hex(), "exact": exact, "magnitude": magnitude})
    g["q4_q8_dots"] = dots

    with open(args.out, "w") as f:
        json.dump(g, f, indent=0)
    print(args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
