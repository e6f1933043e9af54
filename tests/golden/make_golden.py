"""Generates the golden vectors under tests/golden/ by running the reference's own CPU functions.

The reference (createcentury/mamba-metal) keeps its CPU implementation of the scan as NumPy functions
inside its experiment scripts, which import MLX at module level (MLX is not installable here). This
script therefore parses each script with ``ast``, executes only the pure-NumPy function definitions
listed below in a namespace that holds ``np``, and calls them on seeded inputs. Run it in a container
where the reference is mounted (it is not needed, and not present, on the GPU box):

    python tests/golden/make_golden.py /path/to/reference

Functions used (file:line in the reference):
  experiments/09-features/test_features.py  softplus_safe :13, silu :19, reference :23, make_inputs :46
  experiments/10-fp16/test_fp16.py           reference_fp32 :28, make_inputs :58
  experiments/18-prefill/verify_state_out.py reference_h_final :13, main's input draws :30-36
  experiments/07-chunked/selective_scan_chunked.py selective_scan_ref :14, run_test draws :30-35
  experiments/05-pair-scan/pair_scan.py      reference :36, main's input draws :56-81

The reference's feature test seeds each case with ``hash(name)`` (test_features.py:60), which is not
reproducible across Python processes; here each case uses a fixed seed instead (recorded below).
"""

from __future__ import annotations

import ast
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.scan_ref import make_baseline_inputs  # noqa: E402  (seeded BASELINE input generator)


def load_functions(path: Path, names: list[str]) -> dict:
    tree = ast.parse(path.read_text())
    ns: dict = {"np": np}
    found = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            mod = ast.Module(body=[node], type_ignores=[])
            exec(compile(mod, str(path), "exec"), ns)
            found.append(node.name)
    missing = set(names) - set(found)
    if missing:
        raise RuntimeError(f"{path}: functions not found: {missing}")
    return ns


def main(ref_root: Path) -> None:
    exp = ref_root / "experiments"
    feat = load_functions(exp / "09-features/test_features.py", ["softplus_safe", "silu", "reference", "make_inputs"])
    fp16 = load_functions(exp / "10-fp16/test_fp16.py", ["softplus_safe", "silu", "reference_fp32", "make_inputs"])
    state = load_functions(exp / "18-prefill/verify_state_out.py", ["reference_h_final"])
    chunk = load_functions(exp / "07-chunked/selective_scan_chunked.py", ["selective_scan_ref"])
    pair = load_functions(exp / "05-pair-scan/pair_scan.py", ["reference"])
    manifest: dict = {"generator": "tests/golden/make_golden.py", "files": {}}

    def save(name: str, arrays: dict, meta: dict) -> None:
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        manifest["files"][path.name] = {"sha256": hashlib.sha256(path.read_bytes()).hexdigest(), **meta}

    # 1. feature matrix (test_features.py:100-115): same inputs, all flag combinations
    combos = [("baseline", 0, 0, 0), ("D", 1, 0, 0), ("softplus", 0, 0, 1), ("z", 0, 1, 0),
              ("D+z", 1, 1, 0), ("D+softplus", 1, 0, 1), ("all", 1, 1, 1)]
    for tag, (b, d, n, t), seed in (("T1024", (2, 4, 16, 1024), 101), ("T4096", (1, 2, 16, 4096), 102)):
        u, delta, A, B, C, D, z = feat["make_inputs"](b, d, n, t, seed=seed)
        delta_sp = feat["softplus_safe"](delta).copy()
        arrays = dict(u=u, delta=delta, delta_sp=delta_sp, A=A, B=B, C=C, D=D, z=z)
        for name, use_d, use_z, sp in combos:
            if tag == "T4096" and name != "all":
                continue
            arrays[f"y_{name}"] = feat["reference"](u, delta if sp else delta_sp, A, B, C,
                                                    D=D if use_d else None, z=z if use_z else None,
                                                    delta_softplus=bool(sp))
        save(f"features_{tag}", arrays, {"source": "experiments/09-features/test_features.py:23-56,100-115",
                                         "shape": [b, d, n, t], "seed": seed,
                                         "note": "non-softplus cases take delta_sp as delta (test_features.py:63-69)"})

    # 2. fp16 mixed precision (test_fp16.py:110-124): fp32 reference on the unrounded fp32 inputs
    for tag, (b, d, n, t), seed in (("T1024", (2, 4, 16, 1024), 0), ("T4096", (1, 2, 16, 4096), 0)):
        u, delta, A, B, C, D, z = fp16["make_inputs"](b, d, n, t, seed)
        arrays = dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z)
        for name, use_d, use_z, sp in [c for c in combos if c[0] in ("baseline", "D", "z", "softplus", "all")]:
            if tag == "T4096" and name != "all":
                continue
            arrays[f"y_{name}"] = fp16["reference_fp32"](u, delta, A, B, C, D=D if use_d else None,
                                                         z=z if use_z else None, delta_softplus=bool(sp))
        save(f"fp16_{tag}", arrays, {"source": "experiments/10-fp16/test_fp16.py:28-128", "shape": [b, d, n, t],
                                     "seed": seed})

    # 3. final state (verify_state_out.py:30-36): one generator shared across the three shapes
    rng = np.random.default_rng(0)
    arrays = {}
    for i, (b, d, n, t) in enumerate([(1, 2, 8, 256), (2, 4, 16, 1024), (1, 4, 16, 4096)]):
        u = rng.standard_normal((b, d, t)).astype(np.float32)
        delta = rng.uniform(0.01, 0.1, size=(b, d, t)).astype(np.float32)
        A = -rng.uniform(0.1, 2.0, size=(d, n)).astype(np.float32)
        Bw = rng.standard_normal((b, n, t)).astype(np.float32)
        Cw = rng.standard_normal((b, n, t)).astype(np.float32)
        arrays.update({f"u{i}": u, f"delta{i}": delta, f"A{i}": A, f"B{i}": Bw, f"C{i}": Cw,
                       f"h{i}": state["reference_h_final"](u, delta, A, Bw)})
    save("state", arrays, {"source": "experiments/18-prefill/verify_state_out.py:13-49", "cases": 3})

    # 4. chunk boundaries (selective_scan_chunked.py:29-61), seed 0 per case
    arrays = {}
    for i, (b, d, n, t) in enumerate([(1, 2, 8, 512), (1, 2, 8, 1024), (1, 2, 8, 1025), (1, 4, 16, 2048)]):
        rng = np.random.default_rng(0)
        u = rng.standard_normal((b, d, t)).astype(np.float32)
        delta = rng.uniform(0.01, 0.1, size=(b, d, t)).astype(np.float32)
        A = -rng.uniform(0.1, 2.0, size=(d, n)).astype(np.float32)
        Bw = rng.standard_normal((b, n, t)).astype(np.float32)
        Cw = rng.standard_normal((b, n, t)).astype(np.float32)
        arrays.update({f"u{i}": u, f"delta{i}": delta, f"A{i}": A, f"B{i}": Bw, f"C{i}": Cw,
                       f"y{i}": chunk["selective_scan_ref"](u, delta, A, Bw, Cw)})
    save("chunked", arrays, {"source": "experiments/07-chunked/selective_scan_chunked.py:14-61", "cases": 4})

    # 5. pair scan known answers (pair_scan.py:56-81)
    rng = np.random.default_rng(0)
    arrays = {"a0": np.full(1024, 0.5, np.float32), "b0": np.ones(1024, np.float32)}
    arrays["a1"] = rng.uniform(0.0, 1.0, size=1024).astype(np.float32)
    arrays["b1"] = rng.standard_normal(1024).astype(np.float32)
    dl = rng.uniform(0.01, 0.1, size=1024).astype(np.float32)
    uu = rng.standard_normal(1024).astype(np.float32)
    arrays["a2"], arrays["b2"] = np.exp(dl * -1.0).astype(np.float32), (dl * uu).astype(np.float32)
    for i, n in enumerate([33, 100, 513], start=3):
        arrays[f"a{i}"] = rng.uniform(0.0, 1.0, size=n).astype(np.float32)
        arrays[f"b{i}"] = rng.standard_normal(n).astype(np.float32)
    for i in range(6):
        arrays[f"h{i}"] = pair["reference"](arrays[f"a{i}"], arrays[f"b{i}"])
    save("pair_scan", arrays, {"source": "experiments/05-pair-scan/pair_scan.py:36-81", "cases": 6})

    # 6. fp32 (1,16,2048), N=16, D, z, softplus, with the final state
    inp = make_baseline_inputs(1, 16, 16, 2048, seed=0)
    y = feat["reference"](inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], D=inp["D"], z=inp["z"],
                          delta_softplus=True)
    h = state["reference_h_final"](inp["u"], feat["softplus_safe"](inp["delta"]), inp["A"], inp["B"])
    save("config0", {**inp, "y": y, "h": h}, {"source": "BASELINE configs[0]; y via test_features.py:23-43, "
                                                          "state via verify_state_out.py:13-26",
                                               "generator": "oracle.scan_ref.make_baseline_inputs(1,16,16,2048,0)"})

    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout root>")
    main(Path(sys.argv[1]))
