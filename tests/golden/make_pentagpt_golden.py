"""Generate tests/golden/pentagpt_ref.npz by running the REFERENCE's own model.

    python tests/golden/make_pentagpt_golden.py --ref <reference checkout>

(or set PENTANET_REF_DIR).  For each configuration in tests/refmodel.CONFIGS it
builds train_pentagpt.PentaGPT (train_pentagpt.py:101-136) with the
reference's GPTConfig fields set to that size, loads the deterministic weights
of tests/refmodel.weights, and stores, in eval mode on the CPU:
  * the last-position logits of its inference forward in fp32;
  * the same under bf16 autocast (the reference's inference precision; CPU
    autocast here), which sets the scale of bf16 rounding noise;
  * the loss of the targets path (logits at every position) in fp32;
  * the gamma (fp32 mean |W|) the reference computed for each QuantLinear;
  * the logits of tests/refmodel.PentaGPT's fp32 forward, as a check that
    the restatement matches (it is asserted here too).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PENTANET_REF_DIR"),
                    help="the reference checkout (default: $PENTANET_REF_DIR)")
    args = ap.parse_args()
    if not args.ref or not os.path.isfile(os.path.join(args.ref, "train_pentagpt.py")):
        ap.error("pass --ref <reference checkout> (or set PENTANET_REF_DIR)")
    sys.path.insert(0, args.ref)
    sys.path.insert(0, TESTS)
    import train_pentagpt as tp   # the reference module
    import refmodel as rm

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}
    for name, (cfg, seed, batch, seq) in rm.CONFIGS.items():
        gc = tp.GPTConfig(size="small", mode="pentanet", vocab_size=cfg.vocab_size, block_size=cfg.block_size)
        gc.n_layer, gc.n_head, gc.n_embd = cfg.n_layer, cfg.n_head, cfg.n_embd
        ref = tp.PentaGPT(gc).eval()
        mine = rm.PentaGPT(cfg).eval()
        w = rm.weights(mine, seed)
        assert sorted(w) == sorted(ref.state_dict()), "state_dict keys differ from the reference model's"
        ref.load_state_dict(w)
        mine.load_state_dict(w)
        idx, tgt = rm.tokens(cfg, batch, seq, seed)
        with torch.no_grad():
            l32, _ = ref(idx)
            with torch.autocast("cpu", dtype=torch.bfloat16):
                lbf, _ = ref(idx)
            _, loss = ref(idx, tgt)
            lmine, _ = mine(idx)
        d = (lmine - l32).abs().max().item()
        assert d < 1e-4, f"{name}: the restated module differs from the reference by {d}"
        out[f"{name}.logits_f32"] = l32[:, 0].numpy().astype(np.float32)
        out[f"{name}.logits_bf16_autocast"] = lbf[:, 0].float().numpy().astype(np.float32)
        out[f"{name}.loss_f32"] = np.array([loss.item()], dtype=np.float64)
        # the gamma the reference computed for each QuantLinear (named_modules order)
        out[f"{name}.gammas"] = np.array([float(m.weight.abs().mean().clamp(min=1e-8))
                                          for m in rm.quant_layers(ref)], dtype=np.float32)
        print(f"{name}: |restated - ref| {d:.2e}, |bf16 autocast - f32| {(lbf.float() - l32).abs().max():.3f}, "
              f"loss {loss.item():.4f}")
    np.savez_compressed(os.path.join(HERE, "pentagpt_ref.npz"), **out)


if __name__ == "__main__":
    main()
