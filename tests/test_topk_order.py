"""Pin the restated tie order of the CPU ``torch.topk`` (``oracle/topk_order.py``)
against ``torch.topk`` itself, the function the reference's router calls
(``transformers`` ``modeling_qwen3_5_moe.py:767``)."""
import numpy as np
import pytest
import torch

from oracle import topk_order as to


def _torch_ids(x, k):
    return torch.topk(torch.as_tensor(np.asarray(x, dtype=np.float32)), k).indices.tolist()


@pytest.mark.parametrize("n,k,levels", [
    (256, 8, 3), (256, 8, 40), (256, 8, 400), (64, 8, 6), (64, 8, 50), (40, 8, 9),
    (16, 8, 4), (9, 8, 3), (8, 8, 2), (512, 8, 60), (1024, 8, 300), (600, 8, 20),
    (256, 1, 10), (256, 5, 30), (256, 17, 30), (256, 20, 30), (1024, 20, 100)])
def test_restatement_matches_torch_on_ties(n, k, levels):
    rng = np.random.default_rng(n * 1000 + k * 10 + levels)
    for _ in range(60):
        x = (rng.integers(0, levels, size=n) / levels).astype(np.float32)
        assert to.topk_ids(x.tolist(), k) == _torch_ids(x, k)


@pytest.mark.parametrize("n", [16, 40, 64, 100, 256, 257, 512, 1024])
def test_restatement_matches_torch_on_structured_rows(n):
    a = np.arange(n)
    rows = [a, a[::-1], np.r_[a[: n // 2], a[: n - n // 2][::-1]], a % 7, (a * 37) % 11,
            np.zeros(n), a // 2, a[::-1] // 3, np.r_[np.zeros(n - 3), [1, 1, 1]]]
    for r in rows:
        for k in (1, 2, 7, 8, 9):
            x = r.astype(np.float32)
            assert to.topk_ids(x.tolist(), k) == _torch_ids(x, k)


@pytest.mark.parametrize("n", [256, 64, 40])
def test_adversarial_rows_exhaust_the_partition_budget(n, monkeypatch):
    calls = []
    real = to._Row._heap_select

    def spy(self, lo, mid, hi):
        calls.append((lo, mid, hi))
        return real(self, lo, mid, hi)

    row = to.adversarial_row(n, 8)
    monkeypatch.setattr(to._Row, "_heap_select", spy)
    got = to.topk_ids([float(v) for v in row], 8)
    assert calls, "the introselect fallback did not run"
    assert got == _torch_ids(row, 8)


def test_batched_rows_match_torch():
    rng = np.random.default_rng(7)
    x = (rng.integers(0, 25, size=(400, 256)) / 25).astype(np.float32)
    x[:50] = rng.standard_normal((50, 256)).astype(np.float32)   # rows without ties
    ref = torch.topk(torch.from_numpy(x), 8, dim=-1).indices.numpy()
    assert np.array_equal(to.topk_rows(x, 8), ref)


def test_bf16_logit_order_equals_probability_order():
    """The kernels compare model-dtype logits; the reference compares their fp32
    softmax.  On router-like rows both orders agree, ties included."""
    g = torch.Generator().manual_seed(0)
    lg = (torch.randn(2000, 256, generator=g) * 1.1).to(torch.bfloat16)
    p = torch.softmax(lg, dtype=torch.float, dim=-1)
    lf = lg.float()
    for t in range(0, 2000, 7):
        a = lf[t].numpy()
        b = p[t].numpy()
        oa = np.argsort(-a, kind="stable")
        assert np.array_equal(oa, np.argsort(-b, kind="stable"))
        # equal logits <-> equal probabilities
        assert np.array_equal(a[oa][1:] == a[oa][:-1], b[oa][1:] == b[oa][:-1])
