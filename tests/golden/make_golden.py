"""Generate tests/golden/golden.json by running the REFERENCE's own Python code.

Run where a checkout of the reference is available (it is only read):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports the reference's oracles (tests/q4_reference.py, tests/reference_math.py)
and fixture generators (tools/generate_fixtures.py,
tools/generate_q4_matvec_fixtures.py) and records:

* SHA-256 of every reference fixture file (the byte-layout pins);
* dot_q4_q8 of every row of those fixtures (64 / 128 rows, float64 repr);
* reference_head outputs of the three IMROPE fixtures and of seeded
  N(0,1) inputs: SHA-256 of the float64 output bytes plus heads 0 and 31;
* dot_q4_q8 of 32 rows of a seeded benchmark-distribution Q4_K matrix whose
  activation was quantised by this repository's oracle (the reference has no
  quantiser of its own; its dot is what is pinned here).

The JSON is read by tests/test_oracle_golden.py (the oracle against it) and by
the GPU parity tests (test_q4k_gpu.py, test_imrope_gpu.py, test_q8_1_gpu.py,
test_compat_gpu.py); nothing at test time touches the reference checkout.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import platform
import struct
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "golden.json"


def sha(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout (read only)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.dont_write_bytecode = True  # the checkout is read-only
    sys.path[:0] = [str(ref), str(ref / "tests"), str(ref / "tools")]
    import q4_reference  # noqa: E402  (reference tests/q4_reference.py)
    from tests import reference_math  # noqa: E402
    from tools import generate_fixtures  # noqa: E402
    import generate_q4_matvec_fixtures as gq  # noqa: E402

    sys.path.insert(0, str(REPO))
    import oracle  # this repository's oracle: only its quantiser is used here
    from mojo_llm_lab_b200 import fixtures as our_fixtures

    golden = {"python": platform.python_version(),
              "note": "generated from the reference's own Python code; see make_golden.py"}

    # ---------------------------------------------------------------- IMROPE
    imrope = {}
    for name, positions in generate_fixtures.CASES.items():
        fx = generate_fixtures.synthetic_fixture(positions)
        payload = generate_fixtures.serialize_fixture(fx)
        outs = [reference_math.reference_head(row, fx["gamma"], positions) for row in fx["q"]]
        arr = np.array(outs, dtype=np.float64)
        imrope[name] = {"positions": list(positions), "input_sha256": sha(payload),
                        "output_sha256": sha(arr.tobytes()), "head0": arr[0].tolist(),
                        "head31": arr[31].tolist()}
    seeded = {}
    for name, positions in our_fixtures.SEEDED_IMROPE_CASES.items():
        fx = our_fixtures.imrope_seeded_inputs(positions, seed=2024)
        q = fx["q"].astype(np.float64)
        gamma = fx["gamma"].astype(np.float64).tolist()
        outs = [reference_math.reference_head(row.tolist(), gamma, positions) for row in q]
        arr = np.array(outs, dtype=np.float64)
        seeded[name] = {"positions": list(positions), "seed": 2024,
                        "input_sha256": sha(fx["q"].tobytes() + fx["gamma"].tobytes()),
                        "output_sha256": sha(arr.tobytes()), "head0": arr[0].tolist(),
                        "head31": arr[31].tolist()}
    golden["imrope_reference_fixtures"] = imrope
    golden["imrope_seeded"] = seeded
    golden["reference_theta_scale"] = reference_math.BASE ** (-2.0 / reference_math.HEAD_DIM)
    golden["position_axis"] = [reference_math.position_axis(p) for p in range(64)]

    # ---------------------------------------------------------------- Q4
    cases = {
        "default": dict(),
        "random_quants": dict(random_quants=True),
        "gate_up": dict(random_quants=True, gate_up=True),
        "gate_up_rows128": dict(random_quants=True, gate_up=True, rows=128),
        "varied_factors": dict(random_quants=True, gate_up=True, factor_seed=739),
        "varied_activations": dict(random_quants=True, gate_up=True, factor_seed=739,
                                   activation_scale_seed=971),
        "default_activation_scales": dict(activation_scale_seed=971),
        "width2048": dict(random_quants=True, gate_up=True, input_width=2048),
    }
    q4 = {}
    for name, opts in cases.items():
        files = gq.fixtures(**opts)
        width = opts.get("input_width", 2560)
        row_bytes = width // 256 * 144
        acts = files["activations.bin"]
        entry = {"options": opts, "sha256": {k: sha(v) for k, v in files.items()},
                 "bytes": {k: len(v) for k, v in files.items()}}
        for key in ("weights.bin", "gate.bin"):
            if key in files:
                w = files[key]
                entry["dot_" + key.split(".")[0]] = [
                    q4_reference.dot_q4_q8(w[r * row_bytes:(r + 1) * row_bytes], acts)
                    for r in range(len(w) // row_bytes)]
        q4[name] = entry
    golden["q4_reference_fixtures"] = q4

    # Q8_1 known answers: the reference activation blocks re-quantised from
    # their exact float values (x = d * q) must reproduce themselves.
    acts = gq.fixtures()["activations.bin"]
    floats = []
    for start in range(0, len(acts), 36):
        delta, _, *values = struct.unpack_from("<ee32b", acts, start)
        floats.extend(delta * v for v in values)
    golden["q8_1_known_answer"] = {"x": floats, "bytes_sha256": sha(acts)}

    # Seeded benchmark-distribution Q4_K rows through the reference dot.
    k, rows = 2560, 32
    w = our_fixtures.seeded_q4k_matrix(rows, k, seed=11).tobytes()
    x = our_fixtures.seeded_activation(k, seed=12)
    a = oracle.quantize_q8_1(x)
    golden["q4_seeded"] = {
        "rows": rows, "k": k, "weight_seed": 11, "activation_seed": 12,
        "weights_sha256": sha(w), "x_sha256": sha(x.tobytes()), "q8_1_sha256": sha(a),
        "dot": [q4_reference.dot_q4_q8(w[r * 1440:(r + 1) * 1440], a) for r in range(rows)],
    }

    OUT.write_text(json.dumps(golden, indent=1) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
