"""Top-k ids on the device equal the reference's ``torch.topk`` on the CPU, ties included.

Logit rows are planted exactly: token t is the one-hot vector e_t and column t of
the router weight holds row t, so ``logits[t] == rows[t]`` (one exact product).
The rows are chosen to tie often: a few distinct levels, adversarial rows that
use up introselect's partition budget, and E >= 512 (heap-select path).  Every
routing path of the library is covered: the router kernel (T < 128), the
tensor-core router with its top-k kernel (T >= 128), the top-k inside the
decode GEMV (``moe_layer``, T <= 16) and the router kernel feeding the expert
GEMVs (16 < T < 64).  Expected ids come from ``torch.topk`` of the fp32 softmax
on the CPU (the reference's call, modeling_qwen3_5_moe.py:766-767) and from the
oracle's restatement; both must agree with the device, id for id.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from oracle import topk_order as to
from tarfa_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tarfa_b200 import build
    build.build()
    ops.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert ops.device_status() == 0


def planted(rows: np.ndarray, H: int | None = None):
    """bf16 tokens [T, H] and router [E, H] whose exact logits are ``rows``."""
    T, E = rows.shape
    H = H or max(64, (T + 63) // 64 * 64)
    h = torch.zeros(T, H)
    h[torch.arange(T), torch.arange(T)] = 1.0
    w = torch.zeros(E, H)
    w[:, :T] = torch.from_numpy(rows.T.astype(np.float32))
    return h.to(torch.bfloat16), w.to(torch.bfloat16)


def expected(rows: np.ndarray, k: int) -> torch.Tensor:
    lg = torch.from_numpy(rows.astype(np.float32)).to(torch.bfloat16)
    p = torch.softmax(lg, dtype=torch.float, dim=-1)
    ref = torch.topk(p, k, dim=-1).indices
    assert torch.equal(mo.topk_select(p, k), ref)      # the restatement agrees
    return ref


def level_rows(T, E, levels, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, levels, size=(T, E)) * 0.125


def adversarial_rows(E, k, T):
    base = np.array(to.adversarial_row(E, k), dtype=np.float64)
    rows = [base * 0.125]
    rng = np.random.default_rng(E)
    while len(rows) < T:          # the same row under value shifts stays adversarial
        rows.append((base + rng.integers(0, 8)) * 0.125)
    return np.stack(rows[:T])


def _router(rows, k):
    h, w = planted(rows)
    idx, _ = ops.router_topk(h.to(DEV), w.to(DEV), k)
    torch.cuda.synchronize()
    return idx.cpu()


@pytest.mark.parametrize("E,levels", [(256, 3), (256, 12), (256, 60), (64, 4), (64, 20),
                                      (40, 5), (16, 3), (9, 2), (512, 30), (1024, 100)])
def test_router_kernel_tie_order(E, levels):
    for chunk in range(4):                                   # 4 x 16 tokens
        rows = level_rows(16, E, levels, seed=E * 100 + levels * 10 + chunk)
        assert torch.equal(_router(rows, 8), expected(rows, 8)), (E, levels, chunk)


@pytest.mark.parametrize("k", [1, 5, 17, 20, 32])
def test_router_kernel_tie_order_other_k(k):
    rows = level_rows(16, 256, 10, seed=k)
    assert torch.equal(_router(rows, k), expected(rows, k))


@pytest.mark.parametrize("E", [256, 64, 40])
def test_router_kernel_adversarial_rows(E):
    rows = adversarial_rows(E, 8, 16)
    assert torch.equal(_router(rows, 8), expected(rows, 8))


def wide_rows(T, E, seed):
    """A few tokens' worth of close logits, the rest 150 or 300 below: their fp32
    probabilities are exactly 0, ties for the reference though the logits differ."""
    rng = np.random.default_rng(seed)
    rows = np.where(rng.random((T, E)) < 0.5, -150.0, -300.0)
    for t in range(T):
        n = [2, 5, 8, 11][t % 4]
        pos = rng.choice(E, size=n, replace=False)
        rows[t, pos] = rng.integers(0, 4, size=n) * 0.125
    return rows


@pytest.mark.parametrize("E", [256, 64, 1024])
def test_router_kernel_wide_spread(E):
    rows = wide_rows(16, E, seed=E)
    assert torch.equal(_router(rows, 8), expected(rows, 8))


@pytest.mark.parametrize("E,levels,T", [(256, 4, 256), (256, 40, 256), (128, 10, 256), (1024, 50, 256),
                                          (256, 12, 64)])
def test_tensor_core_router_tie_order(E, levels, T):
    rows = level_rows(T, E, levels, seed=E + levels)         # T >= 48: tcgen05 logits + top-k kernel
    if E == 256:
        rows[:16] = adversarial_rows(E, 8, 16)
        rows[16:32] = wide_rows(16, E, seed=3)
    assert torch.equal(_router(rows, 8), expected(rows, 8))


def _layer(E, H=256, I=64, Is=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    sh = [(torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16)
          for s in ((Is, H), (Is, H), (H, Is), (1, H))]
    return gu, dn, sh


@pytest.mark.parametrize("E,T", [(256, 1), (256, 4), (256, 16), (64, 16), (1024, 8), (256, 40)])
def test_moe_layer_tie_order(E, T):
    """Decode batches (T <= 16) route in the router's last CTA, interior tie
    orders settled in the combine; 40 tokens take the router kernel.  The layer
    output follows the same routing as the oracle."""
    rows = level_rows(T, E, 6, seed=E + T)
    if E in (256, 64):
        rows[: min(T, 4)] = adversarial_rows(E, 8, min(T, 4))
    if T >= 8:
        rows[4:8] = wide_rows(4, E, seed=T)
    h, w_r = planted(rows, H=256)
    gu, dn, sh = _layer(E)
    wts = ops.ExpertWeights(gu.to(DEV), dn.to(DEV))
    shd = ops.SharedWeights(*[t.to(DEV) for t in sh])
    out, idx, wt = ops.moe_layer(h.to(DEV), w_r.to(DEV), wts, shd, return_routing=True)
    torch.cuda.synchronize()
    ref_idx = expected(rows, 8)
    assert torch.equal(idx.cpu(), ref_idx)
    idx_o, w_o, _ = mo.router_topk(h, w_r, 8)
    assert torch.equal(idx_o, ref_idx)
    torch.testing.assert_close(wt.cpu(), w_o, rtol=2e-6, atol=0)
    ref = mo.experts_exact(h, idx_o, w_o, lambda e: (gu[e], dn[e]), E) + mo.shared_expert(h, *sh)
    from gpu_helpers import assert_close
    assert_close(out, ref, f"layer on tied routing E={E} T={T}")


@pytest.mark.parametrize("T", [1, 4])
def test_expert_parallel_exchange_tie_order(T):
    """The expert-parallel layer tops-k each token in its exchange kernel: a
    one-rank group (gloo for the handle exchange) returns the oracle's ids in
    order and the single-GPU layer's output."""
    import socket
    import torch.distributed as dist
    from tarfa_b200.ep import EPShard, PeerExpertParallelMoE
    if dist.is_initialized():
        pytest.skip("a process group is already initialised in this process")
    E = 256
    rows = level_rows(T, E, 6, seed=50 + T)
    rows[: min(T, 2)] = adversarial_rows(E, 8, min(T, 2))
    h, w_r = planted(rows, H=256)
    gu, dn, sh = _layer(E)
    wts = ops.ExpertWeights(gu.to(DEV), dn.to(DEV))
    shd = ops.SharedWeights(*[t.to(DEV) for t in sh])
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        ep = PeerExpertParallelMoE(EPShard(w_r.to(DEV), wts, shd, E), max_tokens=8)
        try:
            out, idx, _ = ep.forward(h.to(DEV), return_routing=True)
            ref = ops.moe_layer(h.to(DEV), w_r.to(DEV), wts, shd)
            torch.cuda.synchronize()
            assert ops.device_status() == 0
            assert torch.equal(idx.cpu(), expected(rows, 8))
            assert torch.equal(out, ref)
        finally:
            ep.close()
    finally:
        dist.destroy_process_group()
