"""Qwen3 decoder on B200: the Strassen backend (fused qk_norm_rope / swiglu /
residual epilogues, RMSNorm kernel) against the reference's classical arm
(cuBLAS + unfused math) on the same random weights."""

from __future__ import annotations

import pytest
import torch

from strassen_tpu_b200 import qwen3

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def test_tiny_decoder_strassen_vs_native():
    cfg = qwen3.QWEN3_TINY
    tiles = qwen3.StrassenTiles(bm=256, bk=256, qk_bn=512, up_bn=512, bn=512)
    tp = qwen3.TensorParallel()
    g = torch.Generator().manual_seed(7)
    tokens = torch.randint(0, cfg.vocab, (2, 128), generator=g).cuda()
    ours = qwen3.Qwen3Prefill(cfg, tp, "cuda", backend="strassen", tiles=tiles)
    native = qwen3.Qwen3Prefill(cfg, tp, "cuda", backend="native", tiles=tiles)
    for blk in ours.blocks:
        assert all(site.strassen for site in blk.sites.values()), {k: s.strassen for k, s in blk.sites.items()}
    assert _rel(ours.forward(tokens), native.forward(tokens)) < 5e-2


def test_qwen3_8b_layer_strassen_vs_native():
    cfg = qwen3.QWEN3_8B
    tp = qwen3.TensorParallel()
    tiles = qwen3.StrassenTiles()
    batch, seq = 1, 1024
    ours = qwen3.build_layer(cfg, 0, tp, "cuda", backend="strassen", tiles=tiles)
    native = qwen3.build_layer(cfg, 0, tp, "cuda", backend="native", tiles=tiles)
    assert all(site.strassen for site in ours.sites.values())
    model = qwen3.Qwen3Prefill.__new__(qwen3.Qwen3Prefill)
    model.cfg, model.device, model.blocks = cfg, "cuda", [ours]
    rope = model.rope(batch, seq)
    x = (torch.randn(batch * seq, cfg.hidden, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
         ).to(torch.bfloat16)
    got = qwen3.layer_forward(ours, x, batch, seq, rope)
    want = qwen3.layer_forward(native, x, batch, seq, rope)
    assert torch.isfinite(got.float()).all()
    assert _rel(got - x, want - x) < 3e-2


@pytest.mark.gpu
def test_captured_prefill_replays_the_eager_forward():
    from strassen_tpu_b200 import qwen3
    dev = torch.device("cuda", 0)
    model = qwen3.Qwen3Prefill(qwen3.QWEN3_TINY, qwen3.TensorParallel(), dev, backend="strassen")
    tok = torch.randint(0, qwen3.QWEN3_TINY.vocab, (4, 1024), generator=torch.Generator().manual_seed(3)).to(dev)
    for chunks in (1, 2):
        want = model.forward(tok, chunks=chunks)
        cap = qwen3.CapturedPrefill(model, tok, chunks=chunks)
        got = cap(tok).clone()
        torch.cuda.synchronize()
        cap.release()
        assert torch.equal(got, want)


def test_measured_site_choice_and_mixed_layer():
    """measured_native_sites names only GEMM sites whose native arm it timed faster;
    a layer built with that choice matches the native arm like the all-Strassen one."""
    cfg = qwen3.QWEN3_8B
    tp = qwen3.TensorParallel()
    batch, seq = 1, 2048
    times = qwen3.site_times(cfg, 8, batch * seq, "cuda", steps=3, warmup=1, seq=seq)
    assert set(times) == {"ln1", "q", "k", "v", "attention", "o", "ln2", "up", "down"}
    assert all(t["strassen"] > 0 and t["native"] > 0 for t in times.values())
    assert times["k"]["bn"] == 128 and times["v"]["bn"] == 128  # one-head shards on narrow tiles
    chosen = qwen3.measured_native_sites(cfg, tp, batch * seq, "cuda", seq=seq, steps=3, warmup=1)
    assert chosen <= set(qwen3.GEMM_SITES)
    mixed = qwen3.build_layer(cfg, 0, tp, "cuda", backend="strassen", native_sites=frozenset({"v", "up"}))
    native = qwen3.build_layer(cfg, 0, tp, "cuda", backend="native")
    assert not mixed.sites["v"].strassen and not mixed.sites["up"].strassen and mixed.sites["q"].strassen
    model = qwen3.Qwen3Prefill.__new__(qwen3.Qwen3Prefill)
    model.cfg, model.device, model.blocks = cfg, "cuda", [mixed]
    rope = model.rope(batch, seq)
    x = torch.randn(batch * seq, cfg.hidden, device="cuda", generator=torch.Generator("cuda").manual_seed(4)
                    ).to(torch.bfloat16)
    got = qwen3.layer_forward(mixed, x, batch, seq, rope)
    want = qwen3.layer_forward(native, x, batch, seq, rope)
    assert _rel(got - x, want - x) < 3e-2
