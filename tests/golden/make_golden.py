"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run from the repository root on a machine where the reference tree is mounted:

    python tests/golden/make_golden.py --ref <reference checkout>

(or set PENTANET_REF_DIR to the checkout instead of passing --ref).

It imports the reference's own modules -- ``penta_kernel`` (quantize_and_pack,
unpack_weights, memory_stats; penta_kernel.py:42-106) and ``penta_kernel_cpu``
(numba ``penta_linear_cpu``; penta_kernel_cpu.py:63-101) -- and calls the
reference's AVX2 kernel compiled from ``penta_avx2.c`` by ``oracle/Makefile``
(the reference's shipped binary is never loaded, so ``penta_avx2_wrapper`` is
not imported; its two ctypes calls are restated in ``oracle.ref_avx2_*``).
The int8 line follows penta_avx2_wrapper.py:130-131,137,147 with torch's own
``_int_mm``, applied per token.

Weights and activations are drawn with ``torch.manual_seed`` on the CPU, so the
GPU tests regenerate identical inputs from the recorded seeds; only the
reference outputs (and hashes of the packed bytes) are stored.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gen_weight(N: int, K: int, seed: int, std: float = 0.02) -> torch.Tensor:
    """Config weights: N(0, std) fp32 from torch.manual_seed(seed) on the CPU."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(N, K, generator=g) * std


def gen_act(M: int, K: int, seed: int) -> torch.Tensor:
    """Activations: N(0, 1) fp32 from torch.manual_seed(seed) on the CPU."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g)


def tie_weight(N: int, K: int) -> torch.Tensor:
    """Weights whose w / gamma land exactly on .5 boundaries.  Every row repeats
    (0.5, 1.5, -0.5, -1.5, 2.5, -0.5, 0.5, -0.5, 1.5, 0.5) * 2^-4: mean|w| is
    exactly 2^-4 in any summation order, so round-half-even decides every
    element."""
    base = torch.tensor([0.5, 1.5, -0.5, -1.5, 2.5, -0.5, 0.5, -0.5, 1.5, 0.5]) / 16.0
    reps = (K + 9) // 10
    row = base.repeat(reps)[:K]
    w = row.unsqueeze(0).repeat(N, 1)
    # vary rows by a cyclic shift (keeps the multiset of each full period)
    for n in range(N):
        w[n] = torch.roll(w[n], n % 10)
    return w


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PENTANET_REF_DIR"),
                    help="the reference checkout (default: $PENTANET_REF_DIR)")
    args = ap.parse_args()
    if not args.ref or not os.path.isfile(os.path.join(args.ref, "penta_kernel.py")):
        ap.error("pass --ref <reference checkout> (or set PENTANET_REF_DIR)")
    sys.path.insert(0, args.ref)
    sys.path.insert(0, ROOT)
    import penta_kernel as pk          # reference module
    import penta_kernel_cpu as pkc     # reference module (numba)
    from oracle import oracle as orc

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fixtures: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "reference": "Kyworn/PentaNet-v1.0",
                  "torch": torch.__version__, "cases": {}}

    def record_pack(name: str, w: torch.Tensor, keep_packed: bool) -> tuple:
        packed, K_orig, scale = pk.quantize_and_pack(w)
        p = packed.numpy()
        meta["cases"][name] = {"N": int(w.shape[0]), "K": int(K_orig), "K_packs": int(p.shape[1]),
                               "scale": float(scale), "packed_sha256": sha(p)}
        if keep_packed:
            fixtures[f"{name}.packed"] = p
        unp = pk.unpack_weights(packed, K_orig).numpy()
        meta["cases"][name]["unpacked_sha256"] = sha(unp.astype(np.int8))
        return packed, K_orig, scale

    # ---- config 0: 3072x768 N(0,0.02) seed 0; x (8,768) N(0,1) ------------
    w0 = gen_weight(3072, 768, seed=0)
    packed0, K0, s0 = record_pack("cfg0", w0, keep_packed=False)
    x0 = gen_act(8, 768, seed=100)
    y_numba = pkc.penta_linear_cpu(x0, packed0, s0, K0).numpy()
    w8 = orc.ref_avx2_unpack(packed0.numpy(), K0)
    y_avx2 = orc.ref_avx2_linear(x0.numpy(), w8, s0)
    fixtures["cfg0.y_numba"] = y_numba.astype(np.float32)
    fixtures["cfg0.y_avx2"] = y_avx2.astype(np.float32)
    occ = np.bincount((w8.astype(np.int16) + 2).ravel(), minlength=5) / w8.size
    meta["cases"]["cfg0"].update({"x_seed": 100, "w_seed": 0, "occupancy_m2_to_p2": occ.tolist()})

    # ---- config 1: four GPT-2 shapes, seeds 1..4; x bf16 for M in {1,4,16} --
    shapes = [(768, 2304), (768, 768), (768, 3072), (3072, 768)]   # (K, N)
    for i, (K, N) in enumerate(shapes):
        seed = i + 1
        w = gen_weight(N, K, seed=seed)
        name = f"cfg1.{K}x{N}"
        packed, K_orig, scale = record_pack(name, w, keep_packed=False)
        meta["cases"][name]["w_seed"] = seed
        for M in (1, 4, 16):
            x = gen_act(M, K, seed=1000 + 10 * seed + M).to(torch.bfloat16).float()
            y = pkc.penta_linear_cpu(x, packed, scale, K_orig).numpy()
            fixtures[f"{name}.M{M}.y_numba"] = y.astype(np.float32)
            meta["cases"][name][f"M{M}_x_seed"] = 1000 + 10 * seed + M

    # ---- small / ragged shapes: full packed bytes kept -----------------------
    small = [(1, 1), (1, 7), (3, 10), (5, 13), (17, 25), (64, 96), (33, 161), (128, 770), (7, 1001)]
    for (N, K) in small:
        w = gen_weight(N, K, seed=7 * N + K, std=0.05)
        name = f"small.{N}x{K}"
        packed, K_orig, scale = record_pack(name, w, keep_packed=True)
        meta["cases"][name]["w_seed"] = 7 * N + K
        meta["cases"][name]["std"] = 0.05
        x = gen_act(3, K, seed=N + 3 * K)
        fixtures[f"{name}.y_numba"] = pkc.penta_linear_cpu(x, packed, scale, K_orig).numpy().astype(np.float32)
        meta["cases"][name]["x_seed"] = N + 3 * K

    # ---- round-half-even ties --------------------------------------------------
    wt = tie_weight(12, 50)
    record_pack("ties.12x50", wt, keep_packed=True)
    fixtures["ties.12x50.unpacked"] = pk.unpack_weights(*pk.quantize_and_pack(wt)[:2]).numpy().astype(np.int8)

    # ---- exact roundtrip of random pentanary ints (scripts/benchmark_kernel.py:28-43)
    for (N, K) in [(64, 64), (48, 768)]:
        g = torch.Generator().manual_seed(N * 1000 + K)
        w_true = torch.randint(-2, 3, (N, K), dtype=torch.int32, generator=g)
        name = f"roundtrip.{N}x{K}"
        packed, K_orig, _ = record_pack(name, w_true.float(), keep_packed=True)
        ok = bool((pk.unpack_weights(packed, K_orig) == w_true).all())
        meta["cases"][name]["roundtrip_exact"] = ok
        meta["cases"][name]["w_seed"] = N * 1000 + K

    # ---- int8 line: per-token absmax int8 x, torch._int_mm accumulators ------
    for (M, K, N) in [(8, 96, 64), (16, 770, 48), (5, 33, 20)]:
        w = gen_weight(N, K, seed=M + K + N)
        name = f"int8.{M}x{K}x{N}"
        packed, K_orig, scale = record_pack(name, w, keep_packed=True)
        x = gen_act(M, K, seed=5 * M + K)
        x_scale = x.float().abs().amax(dim=1, keepdim=True) / 127.0        # :130 per row
        x_int8 = (x / x_scale).round().clamp(-128, 127).to(torch.int8)       # :131
        w_int8 = pk.unpack_weights(packed, K_orig).to(torch.int8)
        acc = torch._int_mm(x_int8, w_int8.T.contiguous().T) if M > 16 else \
            (x_int8.to(torch.int64) @ w_int8.to(torch.int64).T).to(torch.int32)
        y = acc.float() * (scale * x_scale)                                   # :147
        fixtures[f"{name}.xq"] = x_int8.numpy()
        fixtures[f"{name}.sx"] = x_scale.squeeze(1).numpy().astype(np.float32)
        fixtures[f"{name}.acc"] = acc.numpy().astype(np.int32)
        fixtures[f"{name}.y"] = y.numpy().astype(np.float32)
        meta["cases"][name].update({"M": M, "x_seed": 5 * M + K, "w_seed": M + K + N})

    # torch._int_mm itself on one shape it supports on CPU (M > 16, K, N multiples of 8)
    M, K, N = 32, 96, 64
    g = torch.Generator().manual_seed(4242)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, generator=g)
    b = torch.randint(-2, 3, (N, K), dtype=torch.int8, generator=g)
    fixtures["intmm.a"] = a.numpy()
    fixtures["intmm.b"] = b.numpy()
    fixtures["intmm.acc"] = torch._int_mm(a, b.T).numpy().astype(np.int32)

    # ---- memory_stats (penta_kernel.py:93-106) ---------------------------------
    meta["memory_stats"] = {f"{N}x{K}": pk.memory_stats(N, K) for (N, K) in
                            [(768, 768), (768, 3072), (3072, 768), (28672, 8192), (1, 1)]}

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **fixtures)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(fixtures), "arrays,", len(meta["cases"]), "cases")


if __name__ == "__main__":
    main()
