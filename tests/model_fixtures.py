"""Synthetic full-size models for the GPU tests: N(0, 0.02) weights drawn on the device
by the Philox kernel (q/k RMSNorm gains 1 + N(0, 0.02)), the way bench.py builds its
model, with an optional host copy of the state dict for the CPU oracle."""

import torch

import ltx_dit

DEV = torch.device("cuda")


def philox_model(cfg: ltx_dit.DiTConfig, seed: int, host_copy: bool = True, dtype=torch.bfloat16):
    """(model, host state dict or None) with the reference's parameter names."""
    with torch.device("meta"):
        model = ltx_dit.LTXModel(cfg)
    gen = ltx_dit.PhiloxGenerator(seed, DEV)
    sd = {}
    for name, p in model.named_parameters():
        w = gen.randn(*p.shape, dtype=dtype).mul_(0.02)
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            w.add_(1.0)
        sd[name] = w
    model.load_state_dict(sd, assign=True)
    host = {k: v.cpu() for k, v in sd.items()} if host_copy else None
    return model.eval(), host
