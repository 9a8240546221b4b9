"""Generate the golden fixtures that pin the CPU oracle.

Run from the repository root in a container that has the reference checkout:

    python tests/golden/gen_golden.py --reference <path-to-rxla-checkout>

Two kinds of fixture come out of it:

1. ``w8_quantizer.npz`` — produced by EXECUTING the reference's own W8 encoder,
   ``benchmarks/quantize_qwen3_5_w8.py`` (``main()``), on a small safetensors
   file.  Its only missing dependency (``typed_args``, an argument parser) is
   replaced by a shim that hands ``main()`` the paths; the tensor code runs
   unmodified under torch.  This pins the U8+128 / f32-scale storage contract.

2. ``reference_known_answers.json`` — the reference's native known-answer tests
   for this path, restated: their literal inputs and their F64 expected values
   (computed here in numpy float64, independently of the C oracle), together
   with each test's tolerance.  Sources (inside the rxla project):
     crates/rxla-core/tests/gqa.rs:32-102
     crates/rxla-core/tests/masked_decode.rs:54-142
     crates/rxla-core/tests/attention.rs (broadcast mask / scales, multihead)
     crates/rxla-core/tests/causal_attention.rs:22-160
     crates/rxla-core/tests/kv_cache.rs:114-172, kv_cache_checked.rs:5-110
     crates/rxla-core/tests/rotary.rs:39-73, rotary_positions.rs:26-100
     crates/rxla-core/tests/layers.rs:44-92
   Literal expected arrays written in those tests are copied as literals.

Nothing under tests/ reads the reference at run time; only this script does.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def f32(a):
    return np.asarray(a, dtype=np.float32)


# --------------------------------------------------------------- W8 encoder

def run_reference_quantizer(reference: Path) -> None:
    import torch
    from safetensors.torch import load_file, save_file

    script = reference / "benchmarks" / "quantize_qwen3_5_w8.py"

    class _Arg:
        def __init__(self, *a, **k):
            pass

    class _TypedArgs:
        _values: dict = {}

        @classmethod
        def parse_args(cls):
            obj = cls.__new__(cls)
            for k, v in cls._values.items():
                setattr(obj, k, v)
            return obj

    shim = types.ModuleType("typed_args")
    shim.Arg = _Arg
    shim.TypedArgs = _TypedArgs
    sys.modules["typed_args"] = shim
    spec = importlib.util.spec_from_file_location("rxla_quantize_w8", script)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    g = torch.Generator().manual_seed(1234)
    tensors = {
        # random rows + edge rows: all-zero row (clamp_min), exact .5 ties, a spike
        "model.language_model.a.weight": torch.randn(6, 256, generator=g) * 0.02,
        "model.language_model.b.weight": torch.randn(5, 128, generator=g),
    }
    a = tensors["model.language_model.a.weight"]
    a[3].zero_()
    a[4] = torch.linspace(-1.0, 1.0, 256)
    a[4, 0] = -1.0
    a[4, 1] = 0.5 * (1.0 / 127.0)   # a tie at 0.5 after scaling
    a[4, 2] = 1.5 * (1.0 / 127.0)   # a tie at 1.5
    a[5, 17] = 40.0                  # one outlier dominates the group scale
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "src.safetensors"
        save_file({k: v.contiguous() for k, v in tensors.items()}, str(src))
        for group in (256, 128, 64, 32):
            if any(v.shape[1] % group for v in tensors.values()):
                continue
            dst = Path(tmp) / f"w8_{group}.safetensors"
            mod.Args._values = {"source": src, "output": dst, "group_size": group}
            mod.main()
            enc = load_file(str(dst))
            for name, v in tensors.items():
                base = name.removesuffix(".weight")
                key = base.split(".")[-1]
                out[f"{key}_g{group}_w"] = v.numpy().astype(np.float32)
                out[f"{key}_g{group}_q"] = enc[name].numpy()
                out[f"{key}_g{group}_s"] = enc[base + ".scale"].numpy()
    np.savez_compressed(HERE / "w8_quantizer.npz", **out)


# --------------------------------------------------------- known answers

def softmax64(logits):
    logits = np.asarray(logits, np.float64)
    m = np.max(logits)
    e = np.exp(logits - m)
    return e / e.sum()


def gqa_case():
    """crates/rxla-core/tests/gqa.rs:32-102"""
    qv = [(i % 9 - 4) / 5 for i in range(48)]
    mask = [float("-inf") if i % 4 == 3 else (i % 7) / 8 for i in range(48)]
    cases = []
    for kv_heads in (1, 2, 4):
        keys = [((i % 11) - 5) / 7 for i in range(2 * kv_heads * 4 * 2)]
        values = [((i % 13) - 6) / 3 for i in range(2 * kv_heads * 4 * 3)]
        qf, kf, vf, mf = f32(qv), f32(keys), f32(values), f32(mask)
        expected = []
        for batch in range(2):
            for head in range(4):
                for row in range(3):
                    kv = head // (4 // kv_heads)
                    logits = []
                    for col in range(4):
                        dot = sum(float(qf[((batch * 4 + head) * 3 + row) * 2 + d]) *
                                  float(kf[((batch * kv_heads + kv) * 4 + col) * 2 + d])
                                  for d in range(2))
                        logits.append(dot / np.sqrt(2.0) + float(mf[(head * 3 + row) * 4 + col]))
                    p = softmax64(logits)
                    for d in range(3):
                        expected.append(sum(p[col] * float(vf[((batch * kv_heads + kv) * 4 + col) * 3 + d])
                                            for col in range(4)))
        cases.append({"kv_heads": kv_heads, "q": qf.tolist(), "k": kf.tolist(), "v": vf.tolist(),
                      "mask": [m if np.isfinite(m) else "-inf" for m in mf.tolist()],
                      "expected": expected})
    return {"source": "crates/rxla-core/tests/gqa.rs:32-102", "tolerance": 2e-6,
            "q_shape": [2, 4, 3, 2], "mask_shape": [1, 4, 3, 4], "cases": cases}


def masked_decode_case():
    """crates/rxla-core/tests/masked_decode.rs:54-142 (cache [2,4,2], 4 steps)"""
    steps = []
    keys, values = [], []
    for step in range(4):
        s = float(step)
        q = f32([0.5 + s / 4, -0.25, 0.75, 0.1 + s / 3])
        k = f32([s / 2, 0.5, 1 - s / 3, -0.25])
        v = f32([s + 1, -s, 2 * s, 0.25 + s])
        keys.append(k)
        values.append(v)
        out, probs = [], []
        for head in range(2):
            logits = [sum(float(q[head * 2 + d]) * float(key[head * 2 + d]) for d in range(2)) / np.sqrt(2.0)
                      for key in keys]
            p = softmax64(logits)
            for d in range(2):
                out.append(sum(float(val[head * 2 + d]) * p[t] for t, val in enumerate(values)))
            probs.extend([p[t] if t <= step else 0.0 for t in range(4)])
        steps.append({"q": q.tolist(), "k": k.tolist(), "v": v.tolist(), "position": step,
                      "expected_out": out, "expected_probs": probs})
    return {"source": "crates/rxla-core/tests/masked_decode.rs:54-142", "tolerance": 2e-6,
            "prob_tolerance": 1e-6, "cache_shape": [2, 4, 2], "cache_k_init": 100.0,
            "cache_v_init": 1000.0, "steps": steps}


def attention_cases():
    """crates/rxla-core/tests/attention.rs: broadcast mask + explicit scales; multihead."""
    bias = float(np.float32(np.log(2.0)))
    first = {"q": [1, 0, 1, 0], "k": [1, 0, 0, 0, 0, 1], "v": [3, 6, 1000, 9, 12, 1000],
             "mask": [0.0, bias, "-inf"], "scales": [0.0, -1.0], "expected": []}
    b = np.exp(np.float64(np.float32(bias)))
    for scale in (0.0, -1.0):
        a = np.exp(scale)
        first["expected"].append([(f * a + s * b) / (a + b) for f, s in ((3, 6), (9, 12))])
    qv = f32([((i * 7 % 19) - 9) / 8 for i in range(48)])
    kv = f32([((i * 3 % 17) - 8) / 7 for i in range(60)])
    vv = f32([((i * 11 % 23) - 11) / 6 for i in range(60)])
    ey, ep = [], []
    for bh in range(6):
        for query in range(4):
            logits = [sum(float(qv[bh * 8 + query * 2 + d]) * float(kv[bh * 10 + key * 2 + d])
                          for d in range(2)) / np.sqrt(2.0) for key in range(5)]
            p = softmax64(logits)
            for d in range(2):
                ey.append(sum(p[key] * float(vv[bh * 10 + key * 2 + d]) for key in range(5)))
            ep.extend(p.tolist())
    multi = {"q": qv.tolist(), "k": kv.tolist(), "v": vv.tolist(), "shape_q": [2, 3, 4, 2],
             "shape_k": [2, 3, 5, 2], "expected_y": ey, "expected_p": ep}
    return {"source": "crates/rxla-core/tests/attention.rs:96-190", "tolerance": 2e-6,
            "broadcast": first, "multihead": multi}


def causal_cases():
    """crates/rxla-core/tests/causal_attention.rs:22-160 (literal expectations)"""
    qv = f32([(i - 3) * 0.125 for i in range(10)])
    kv = f32([(i - 6) * 0.125 for i in range(14)])
    vv = f32([(i - 5) * 0.25 for i in range(14)])
    full = []
    for i in range(5):
        scores = [np.exp(sum(float(qv[i * 2 + d]) * float(kv[j * 2 + d]) for d in range(2)))
                  for j in range(i + 1)]
        tot = sum(scores)
        for d in range(2):
            full.append(sum(s / tot * float(vv[j * 2 + d]) for j, s in enumerate(scores)))
    return {
        "source": "crates/rxla-core/tests/causal_attention.rs:22-160",
        "tolerance": 2e-5,
        "runtime_positions": {
            "keys": [0, 1, 2, 3], "values": [10.0, 20.0, 30.0, 40.0],
            "cases": [{"q": [0, 2], "expected": [10.0, 20.0]},
                      {"q": [1, 3], "expected": [15.0, 25.0]}],
        },
        "extreme_positions": {
            "q": [16777216, 2147483647],
            "k": [16777216, 16777217, 2147483647, -2147483648],
            "expected": [0.0, "-inf", "-inf", 0.0, 0.0, 0.0, 0.0, 0.0],
        },
        "offset_mask": {"queries": 2, "keys": 4, "offset": 1,
                        "expected": [0.0, 0.0, "-inf", "-inf", 0.0, 0.0, 0.0, "-inf"]},
        "full": {"q": qv.tolist(), "k": kv.tolist(), "v": vv.tolist(), "expected": full,
                 "chunks": [[0, 2], [2, 5], [4, 5]]},
    }


def kv_cases():
    """crates/rxla-core/tests/kv_cache.rs:114-172 and kv_cache_checked.rs:5-110"""
    checked_steps = []
    ek = [0.0] * 8
    ev = [0.0] * 8
    for step, (row, col, valid) in enumerate([(0, 0, True), (-1, 0, False), (3, 0, False),
                                              (2, 0, True), (1, 1, False),
                                              (2147483647, 0, False), (1, 0, True)]):
        data = [step + 1.0] * 4 if valid else ["nan"] * 4
        vals = [-(step + 1.0)] * 4 if valid else ["inf"] * 4
        if valid:
            ek[row * 2:row * 2 + 4] = data
            ev[row * 2:row * 2 + 4] = [-(step + 1.0)] * 4
        checked_steps.append({"row": row, "col": col, "valid": valid, "k": data, "v": vals,
                              "expected_k": list(ek), "expected_v": list(ev)})
    return {
        "source": "crates/rxla-core/tests/kv_cache.rs:114-172, kv_cache_checked.rs:5-110",
        "clamp": {"cache_shape": [3, 1],
                  "updates": [[-5, 1.0, 10.0], [99, 3.0, 30.0], [1, 2.0, 20.0]],
                  "expected_k": [1.0, 2.0, 3.0], "expected_v": [10.0, 20.0, 30.0]},
        "checked": {"cache_shape": [4, 2], "update_shape": [2, 2], "steps": checked_steps},
    }


def rotary_cases():
    """crates/rxla-core/tests/rotary.rs:39-73 and rotary_positions.rs:26-100"""
    values = f32([(i - 12) / 3 for i in range(24)])
    tables = []
    for offset in (0.0, 0.7):
        angles = f32([i / 5 + offset for i in range(6)])
        cos = np.cos(angles).astype(np.float32)
        sin = np.sin(angles).astype(np.float32)
        exp = {}
        for layout in (0, 1):
            e = [0.0] * 24
            for row in range(6):
                for pair in range(2):
                    a, b = (pair, pair + 2) if layout == 0 else (pair * 2, pair * 2 + 1)
                    c = float(cos[(row % 3) * 2 + pair])
                    s = float(sin[(row % 3) * 2 + pair])
                    av, bv = float(values[row * 4 + a]), float(values[row * 4 + b])
                    e[row * 4 + a] = av * c - bv * s
                    e[row * 4 + b] = bv * c + av * s
            exp[str(layout)] = e
        tables.append({"cos": cos.tolist(), "sin": sin.tolist(), "expected": exp})
    pos_cases = []
    vals2 = f32([(i - 10) * 0.25 for i in range(24)])
    for positions, freqs in (([0.0, 1.0, 3.0], [0.125, 0.5]), ([2.0, 4.0, 5.0], [0.25, -0.125])):
        exp = {}
        for layout in (0, 1):
            e = [0.0] * 24
            for batch in range(2):
                for p, position in enumerate(positions):
                    for fi, freq in enumerate(freqs):
                        base = (batch * 3 + p) * 4
                        a, b = (base + fi, base + fi + 2) if layout == 0 else (base + 2 * fi, base + 2 * fi + 1)
                        ang = float(np.float32(position)) * float(np.float32(freq))
                        s, c = np.sin(ang), np.cos(ang)
                        va, vb = float(vals2[a]), float(vals2[b])
                        e[a] = va * c - vb * s
                        e[b] = vb * c + va * s
            exp[str(layout)] = e
        pos_cases.append({"positions": positions, "frequencies": freqs, "expected": exp})
    return {"source": "crates/rxla-core/tests/rotary.rs:39-73, rotary_positions.rs:26-100",
            "tolerance": 1e-6, "position_tolerance": 5e-6, "values": values.tolist(),
            "tables": tables, "values_positions": vals2.tolist(), "position_cases": pos_cases}


def linear_cases():
    """crates/rxla-core/tests/layers.rs:44-92 (rel tol 3e-5)"""
    out = []
    for shape in ([3], [2, 3], [2, 2, 3]):
        rows = int(np.prod(shape)) // 3
        vals = [float(i - 2) for i in range(rows * 3)]
        exp = []
        for r in range(rows):
            v = vals[r * 3:r * 3 + 3]
            exp += [v[0] - 2 * v[1] + 3 * v[2], 4 * v[0] - v[2]]
        out.append({"shape": shape, "x": vals, "expected": exp,
                    "expected_bias": [e + (0.5 if i % 2 == 0 else -1.0) for i, e in enumerate(exp)]})
    return {"source": "crates/rxla-core/tests/layers.rs:44-92", "rel_tolerance": 3e-5,
            "weight": [1.0, -2.0, 3.0, 4.0, 0.0, -1.0], "bias": [0.5, -1.0], "cases": out}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    run_reference_quantizer(args.reference)
    fixture = {
        "gqa": gqa_case(),
        "masked_decode": masked_decode_case(),
        "attention": attention_cases(),
        "causal": causal_cases(),
        "kv_cache": kv_cases(),
        "rotary": rotary_cases(),
        "linear": linear_cases(),
    }
    with open(HERE / "reference_known_answers.json", "w") as f:
        json.dump(fixture, f, indent=1)
    print("wrote", HERE / "reference_known_answers.json", HERE / "w8_quantizer.npz")


if __name__ == "__main__":
    main()
