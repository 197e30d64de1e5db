#!/usr/bin/env python3
"""Regenerates the golden fixtures in this folder from the reference's OWN Python oracles.

Run here (where the math-plus checkout is mounted), never on the GPU box:

    python tests/golden/make_golden.py --reference <checkout of johnhenry/math-plus>

It drives, as subprocesses and through their documented stdin/job-file interfaces:

* packages/tensor-webgpu/scripts/gemm_oracle.py       (C = A@B and |A|@|B| in f64)
* packages/tensor-webgpu/scripts/attention_oracle.py  (masked softmax attention in f64)
* packages/tensor-cpu/scripts/numpy_oracle.py         (linear / matmul / sdpa / softmax / gelu /
                                                       rope / geglu / mean_pool / sort / gather_rows)
* packages/special/scripts/special_oracle.py          (SciPy erf / erfc / x*ndtr(x))

Inputs come from the reference tests' own generators, restated here in pure
Python (independently of oracle/mp_oracle.c, so the fixture also pins the C
restatement of the generators through the stored input prefixes):

* gemm.test.ts:85-93 and flash-attention.test.ts:49-57 LCG, seeds per
  gemm.test.ts:109-112 / flash-attention.test.ts makeCase;
* tensor-cpu/test/helpers.ts:115-124 ``seeded`` LCG.

Outputs are written to gemm_webgpu.npz, attention_webgpu.npz,
differential_cpu.npz and special.npz next to this script.
"""
from __future__ import annotations

import argparse
import base64
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


# ---- the reference tests' input generators, restated in pure Python ----------------------

def lcg_webgpu(size: int, seed: int) -> np.ndarray:
    """gemm.test.ts:85-93 / flash-attention.test.ts:49-57, stored into a Float32Array."""
    s = seed & 0xFFFFFFFF
    out = np.empty(size, np.float64)
    for i in range(size):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = (s / 0xFFFFFFFF) * 2 - 1
    return out.astype(np.float32)


def lcg_seeded(n: int, seed: int, lo: float = -2.0, hi: float = 2.0) -> np.ndarray:
    """tensor-cpu/test/helpers.ts:115-124 (f64 values)."""
    s = (seed & 0xFFFFFFFF) or 1
    out = np.empty(n, np.float64)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = lo + ((s >> 8) / 2**24) * (hi - lo)
    return out


def b64(a: np.ndarray) -> str:
    return base64.b64encode(np.ascontiguousarray(a).tobytes()).decode("ascii")


def unb64(s: str, dtype) -> np.ndarray:
    return np.frombuffer(base64.b64decode(s), dtype=dtype).copy()


# ---- GEMM: packages/tensor-webgpu/test/gemm.test.ts ---------------------------------------

# gemm.test.ts:147-163. "full" shapes keep every output; the rest keep a 256-entry sample.
GEMM_SHAPES = [
    (4, 3, 5, False, "full"), (17, 33, 9, False, "full"), (128, 128, 128, False, "sample"),
    (1, 64, 256, False, "full"), (37, 70, 45, True, "full"), (1, 1024, 300, True, "full"),
    (33, 256, 100, True, "full"), (50, 128, 96, True, "full"), (65, 64, 64, True, "full"),
    (93, 256, 200, True, "sample"), (300, 268, 130, True, "sample"), (130, 256, 200, False, "sample"),
    (257, 100, 132, False, "sample"), (130, 256, 202, False, "sample"), (256, 512, 256, False, "sample"),
]


def gemm_fixtures(ref: str) -> dict:
    script = os.path.join(ref, "packages/tensor-webgpu/scripts/gemm_oracle.py")
    cases, meta = [], []
    for dtype in ("f32", "f16"):
        for (m, k, n, trans_b, keep) in GEMM_SHAPES:
            seed = m * 7919 + k * 104729 + n * 1299709 + (17 if trans_b else 0)  # gemm.test.ts:109-112
            a = lcg_webgpu(m * k, seed)
            b = lcg_webgpu(k * n, seed + 1)
            if dtype == "f16":
                ab, bb = a.astype(np.float16), b.astype(np.float16)  # Float16Array.from: RNE
            else:
                ab, bb = a, b
            cases.append({"a": b64(ab), "b": b64(bb), "dtype": dtype, "m": m, "k": k, "n": n, "transB": trans_b})
            meta.append((dtype, m, k, n, trans_b, keep, seed, a, b))
    out = subprocess.run([sys.executable, script], input=json.dumps({"cases": cases}), capture_output=True,
                         text=True, check=True).stdout
    results = json.loads(out)["results"]
    fx = {}
    rng = np.random.default_rng(20261201)
    for (dtype, m, k, n, trans_b, keep, seed, a, b), r in zip(meta, results):
        key = f"{dtype}_{m}x{k}x{n}_{'T' if trans_b else 'N'}"
        c = unb64(r["c"], "<f8")
        p = unb64(r["absprod"], "<f8")
        fx[key + "_seed"] = np.array([seed], np.int64)
        fx[key + "_aprefix"] = a[:8].copy()
        fx[key + "_bprefix"] = b[:8].copy()
        if keep == "full":
            fx[key + "_idx"] = np.arange(m * n, dtype=np.int64)
        else:
            fx[key + "_idx"] = np.sort(rng.choice(m * n, size=256, replace=False)).astype(np.int64)
        idx = fx[key + "_idx"]
        fx[key + "_c"] = c[idx]
        fx[key + "_absprod"] = p[idx]
    return fx


# ---- attention: packages/tensor-webgpu/test/flash-attention.test.ts ---------------------

def sliding_window(lq, lk, radius):
    m = np.zeros(lq * lk, np.float32)
    for i in range(lq):
        c = int(np.floor((i * (lk - 1)) / max(1, lq - 1) + 0.5))  # Math.round
        for j in range(max(0, c - radius), min(lk - 1, c + radius) + 1):
            m[i * lk + j] = 1
    return m


def padding(batch, lk, lens):
    m = np.zeros(batch * lk, np.float32)
    for b in range(batch):
        m[b * lk: b * lk + lens[b]] = 1
    return m


def causal(lq, lk):
    m = np.zeros(lq * lk, np.float32)
    for i in range(lq):
        m[i * lk: i * lk + min(i, lk - 1) + 1] = 1
    return m


def random_mask(batch, lq, lk, seed):
    r = lcg_webgpu(batch * lq * lk, seed)
    m = (r > 0.4).astype(np.float32)
    m[(1 * lq + 3) * lk:(1 * lq + 4) * lk] = 0
    return m


# flash-attention.test.ts:257-336 (name, B, LQ, LK, D, scale or None, mask kind, seed)
ATTN_CASES = [
    ("d64_unmasked", 2, 37, 45, 64, None, None, 1),
    ("d32_unmasked_odd_scale", 1, 5, 3, 32, 0.7, None, 4),
    ("d32_sliding_window", 2, 40, 70, 32, None, ("window", 6), 7),
    ("d48_random_mask_full_row", 2, 20, 50, 48, None, ("random", 99), 10),
    ("d64_key_padding", 3, 33, 90, 64, None, ("padding", [90, 50, 17]), 13),
    ("d128_causal", 2, 40, 40, 128, None, ("causal",), 19),
    ("d5_unmasked", 2, 9, 11, 5, 0.7, None, 22),
    ("d32_padding_broadcast", 2, 17, 64, 32, None, ("padding1", [30]), 25),
]


def attention_fixtures(ref: str) -> dict:
    script = os.path.join(ref, "packages/tensor-webgpu/scripts/attention_oracle.py")
    cases, metas = [], []
    for (name, B, LQ, LK, D, scale, mk, seed) in ATTN_CASES:
        q = lcg_webgpu(B * LQ * D, seed)
        k = lcg_webgpu(B * LK * D, seed + 1)
        v = lcg_webgpu(B * LK * D, seed + 2)
        sc = scale if scale is not None else 1 / np.sqrt(D)
        mask, mshape = None, None
        if mk is not None:
            if mk[0] == "window":
                mask, mshape = sliding_window(LQ, LK, mk[1]), [LQ, LK]
            elif mk[0] == "random":
                mask, mshape = random_mask(B, LQ, LK, mk[1]), [B, LQ, LK]
            elif mk[0] == "padding":
                mask, mshape = padding(B, LK, mk[1]), [B, 1, LK]
            elif mk[0] == "padding1":
                mask, mshape = padding(1, LK, mk[1]), [LK]
            elif mk[0] == "causal":
                mask, mshape = causal(LQ, LK), [LQ, LK]
        cases.append({"q": b64(q), "k": b64(k), "v": b64(v), "batch": B, "seqQ": LQ, "seqK": LK, "dim": D,
                      "scale": float(sc), "mask": b64(mask) if mask is not None else None, "maskShape": mshape})
        metas.append((name, B, LQ, LK, D, sc, seed, q, mask, mshape))
    out = subprocess.run([sys.executable, script], input=json.dumps({"cases": cases}), capture_output=True,
                         text=True, check=True).stdout
    results = json.loads(out)["results"]
    fx = {}
    for (name, B, LQ, LK, D, sc, seed, q, mask, mshape), r in zip(metas, results):
        fx[name + "_dims"] = np.array([B, LQ, LK, D, seed], np.int64)
        fx[name + "_scale"] = np.array([sc], np.float64)
        fx[name + "_qprefix"] = q[:8].copy()
        if mask is not None:
            fx[name + "_mask"] = mask
            fx[name + "_maskshape"] = np.array(mshape, np.int64)
        fx[name + "_out"] = unb64(r["out"], "<f8")
    return fx


# ---- tensor-cpu differential cases: packages/tensor-cpu/test/differential.test.ts -------

def differential_fixtures(ref: str) -> dict:
    """linear / matmul / sdpa / softmax / gelu / rope / geglu / meanPool / sort / gatherRows cases from
    differential.test.ts:96-160, through numpy_oracle.py."""
    script = os.path.join(ref, "packages/tensor-cpu/scripts/numpy_oracle.py")
    counter = [0]

    def f32(shape, lo=-2.0, hi=2.0):
        counter[0] += 1
        seed = 7919 * counter[0]
        n = int(np.prod(shape))
        return seed, lo, hi, lcg_seeded(n, seed, lo, hi).astype(np.float32).reshape(shape)

    def boolean(shape, p):
        counter[0] += 1
        seed = 15485863 * counter[0]
        n = int(np.prod(shape))
        return seed, p, (lcg_seeded(n, seed, 0, 1) < p).astype(np.bool_).reshape(shape)

    def pad_mask(B, Lk):
        seed, p, m = boolean((B, 1, 1, Lk), 0.7)
        m = m.copy()
        m[:, 0, 0, 0] = True
        return seed, p, m

    def causal_mask(L):
        return np.array([[(k <= i) for k in range(L)] for i in range(L)], np.bool_).reshape(1, 1, L, L)

    cases = []

    def add(name, op, args, tensors, gen):
        cases.append((name, op, args, tensors, gen))

    def linear_case(name, xs, ws, bias):
        x, w = f32(xs), f32(ws)
        tensors, gen = [x[3], w[3]], [x[:3], w[:3]]
        if bias:
            b = f32((ws[0],))
            tensors.append(b[3])
            gen.append(b[:3])
        add(name, "linear", {}, tensors, gen)

    linear_case("linear_2x37x96_w70_bias", (2, 37, 96), (70, 96), True)
    linear_case("linear_300x33_w67", (300, 33), (67, 33), False)
    a, b = f32((2, 1, 5, 7)), f32((3, 7, 6))
    add("matmul_2x1x5x7_3x7x6", "matmul", {}, [a[3], b[3]], [a[:3], b[:3]])
    a, b = f32((65, 9)), f32((9, 69))
    add("matmul_65x9_9x69", "matmul", {}, [a[3], b[3]], [a[:3], b[:3]])

    def sdpa_case(name, B, H, Hk, Lq, Lk, D, mask):
        q, k, v = f32((B, H, Lq, D)), f32((B, Hk, Lk, D)), f32((B, Hk, Lk, D))
        tensors, gen = [q[3], k[3], v[3]], [q[:3], k[:3], v[:3]]
        if mask is not None:
            tensors.append(mask)
        add(name, "sdpa", {"scale": 1 / np.sqrt(D)}, tensors, gen)

    sdpa_case("sdpa_gqa_h4_hk2", 2, 4, 2, 9, 9, 8, None)
    pm = pad_mask(2, 11)
    sdpa_case("sdpa_gqa_h6_hk1_pad", 2, 6, 1, 5, 11, 16, pm[2])
    sdpa_case("sdpa_causal_13", 1, 3, 3, 13, 13, 8, causal_mask(13))
    add_mask = f32((1, 2, 7, 7), -3, 1)
    sdpa_case("sdpa_additive", 1, 2, 2, 7, 7, 4, add_mask[3])
    pm2 = pad_mask(1, 128)
    sdpa_case("sdpa_encoder_b1_h16_l128_d64", 1, 16, 16, 128, 128, 64, pm2[2])
    x = f32((3, 6, 5), -40, 40)
    add("softmax_mid_axis", "softmax", {"axis": 1}, [x[3]], [x[:3]])
    x = f32((200,), -10, 10)
    add("gelu_200", "unary", {"fn": "gelu"}, [x[3]], [x[:3]])
    # differential.test.ts:109-116, 153, 160: rope, geglu, meanPool, sort, gatherRows
    x = f32((1, 3, 17, 16))
    add("rope_base10000_1x3x17x16", "rope", {"base": 10000.0}, [x[3]], [x[:3]])
    x = f32((2, 2, 70, 32))
    add("rope_base160000_2x2x70x32", "rope", {"base": 160000.0}, [x[3]], [x[:3]])
    x = f32((3, 5, 24), -6, 6)
    add("geglu_3x5x24", "geglu", {}, [x[3]], [x[:3]])
    x = f32((3, 7, 5))
    pool_mask = np.array([1, 1, 0, 1, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1], np.bool_).reshape(3, 7)
    add("mean_pool_3x7x5", "mean_pool", {}, [x[3], pool_mask], [x[:3]])
    x = f32((5, 3))
    add("sort_axis0_5x3", "sort", {"axis": 0}, [x[3]], [x[:3]])
    x = f32((2, 7, 3))
    counter[0] += 1
    gather_idx = np.floor(lcg_seeded(8, 104729 * counter[0], -7, 7)).astype(np.int32).reshape(2, 4)
    add("gather_rows_2x7x3_idx2x4", "gather_rows", {}, [x[3], gather_idx], [x[:3]])

    fx = {}
    with tempfile.TemporaryDirectory() as d:
        jobs = []
        for i, (name, op, args, tensors, gen) in enumerate(cases):
            paths = []
            for j, t in enumerate(tensors):
                p = os.path.join(d, f"in-{i}-{j}.npy")
                np.save(p, t)
                paths.append(p)
            jobs.append({"op": op, "inputs": paths, "args": {k: float(v) if isinstance(v, (float, np.floating)) else v
                                                             for k, v in args.items()},
                         "output": os.path.join(d, f"out-{i}.npy")})
        jp = os.path.join(d, "jobs.json")
        with open(jp, "w") as f:
            json.dump(jobs, f)
        subprocess.run([sys.executable, script, jp], check=True)
        for i, (name, op, args, tensors, gen) in enumerate(cases):
            fx[name + "_out"] = np.load(os.path.join(d, f"out-{i}.npy"))
            fx[name + "_gen"] = np.array([[s, lo, hi] for (s, lo, hi) in gen], np.float64)
            fx[name + "_shapes"] = np.array([list(t.shape) + [0] * (4 - t.ndim) for t in tensors], np.int64)
            fx[name + "_ranks"] = np.array([t.ndim for t in tensors], np.int64)
            if op == "sdpa" and len(tensors) > 3:
                fx[name + "_mask"] = tensors[3]
            if op == "mean_pool":
                fx[name + "_mask"] = tensors[1]
            if op == "gather_rows":
                fx[name + "_idx"] = tensors[1]
            if "base" in args:
                fx[name + "_base"] = np.array([args["base"]], np.float64)
            if "scale" in args:
                fx[name + "_scale"] = np.array([args["scale"]], np.float64)
            if "axis" in args:
                fx[name + "_axis"] = np.array([args["axis"]], np.int64)
            fx[name + "_prefix0"] = tensors[0].reshape(-1)[:8].astype(np.float32)
    fx["_names"] = np.array([c[0] for c in cases])
    return fx


# ---- special functions: packages/special/test/special-oracle.test.ts ---------------------

def special_fixtures(ref: str) -> dict:
    script = os.path.join(ref, "packages/special/scripts/special_oracle.py")
    # The grids of special-oracle.test.ts:76 (erf, [-6, 6] step 1/256), :87 (both erfc tails,
    # step 1/16 out to 27.25) and :92 (GELU, [-38, 12] step 1/16).
    dense = np.arange(-6 * 256, 6 * 256 + 1) / 256
    tails = np.arange(6 * 16, int(27.25 * 16) + 1) / 16
    xs = np.concatenate([dense, tails, -tails])
    gx = np.arange(-38 * 16, 12 * 16 + 1) / 16
    fx = {"erf_x": xs, "gelu_x": gx}
    with tempfile.TemporaryDirectory() as d:
        for op, x in (("erf", xs), ("erfc", xs), ("gelu_ndtr", gx)):
            jp = os.path.join(d, "job.json")
            with open(jp, "w") as f:
                json.dump({"op": op, "xs": [float(v) for v in x]}, f)
            out = subprocess.run([sys.executable, script, jp], capture_output=True, text=True, check=True).stdout
            fx[op] = np.array(json.loads(out), np.float64)
    return fx


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of the reference repository (johnhenry/math-plus)")
    ap.add_argument("--only", choices=["gemm", "attention", "differential", "special"],
                    help="regenerate one fixture file")
    args = ap.parse_args()
    ref = args.reference
    makers = {"gemm": ("gemm_webgpu.npz", gemm_fixtures), "attention": ("attention_webgpu.npz", attention_fixtures),
              "differential": ("differential_cpu.npz", differential_fixtures),
              "special": ("special.npz", special_fixtures)}
    for key, (fname, make) in makers.items():
        if args.only in (None, key):
            np.savez_compressed(os.path.join(HERE, fname), **make(ref))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
