"""Helpers shared by the GPU parity tests (no GPU needed to import)."""
import torch
import torch.nn.functional as F

# Tolerance for model-dtype outputs of the expert path, written into every test:
# max |out - ref| <= 2^-7 * max |ref|  and  cosine(out, ref) >= 0.99999.
REL_MAX = 2.0 ** -7
COS_MIN = 0.99999


def close_report(out: torch.Tensor, ref: torch.Tensor):
    o = out.detach().float().cpu().flatten()
    r = ref.detach().float().cpu().flatten()
    err = (o - r).abs().max().item() if o.numel() else 0.0
    scale = r.abs().max().item() if r.numel() else 0.0
    cos = F.cosine_similarity(o.double(), r.double(), dim=0).item() if r.abs().sum() > 0 else 1.0
    exact = (out.detach().cpu() == ref.detach().cpu()).float().mean().item() if o.numel() else 1.0
    return err, scale, cos, exact


def assert_close(out: torch.Tensor, ref: torch.Tensor, what: str = ""):
    err, scale, cos, exact = close_report(out, ref)
    assert err <= REL_MAX * scale + 1e-30, f"{what}: max err {err} > 2^-7 * {scale}"
    assert cos >= COS_MIN, f"{what}: cosine {cos} < {COS_MIN}"
    return exact
