"""The configuration-5 language model built on the FirstPassageAttention layer: shape, one training step, and the
native kernels against the reference attention inside the full model."""
import math

import pytest
import torch

from first_passage_attention_b200.lm import FPALanguageModel, LMConfig, LMTrainer, make_tokens


def test_config5_parameter_count():
    with torch.device("meta"):
        m = FPALanguageModel(LMConfig())
    d, v, L, H = 768, 50304, 12, 12
    per_block = (d * 3 * d) + (d * d) + (d * 3 * H + 3 * H + H) + 2 * 2 * d + (d * 4 * d + 4 * d) + (4 * d * d + d)
    assert m.n_params() == v * d + L * per_block + 2 * d
    assert 1.0e8 < m.n_params() < 1.3e8  # "110M-param GPT-2-small-shaped"


def test_tiny_model_trains_on_cpu_with_reference_attention():
    torch.manual_seed(0)
    cfg = LMConfig(vocab=97, d_model=32, n_heads=2, n_layers=2)
    model = FPALanguageModel(cfg, impl="reference")
    tr = LMTrainer(model, lr=3e-3, ddp=False)
    tok = make_tokens(2, 16, cfg.vocab, seed=1, device="cpu")
    first = tr.step(tok).item()
    assert math.isfinite(first) and abs(first - math.log(cfg.vocab)) < 0.5
    for _ in range(30):
        last = tr.step(tok).item()
    assert last < first - 0.5  # memorises the fixed batch


@pytest.mark.gpu
def test_lm_native_matches_reference_attention_and_trains():
    torch.manual_seed(0)
    cfg = LMConfig(vocab=512, d_model=128, n_heads=2, n_layers=2)
    dev = torch.device("cuda")
    native = FPALanguageModel(cfg).to(dev)
    ref = FPALanguageModel(cfg, impl="reference").to(dev)
    ref.load_state_dict(native.state_dict())
    tok = make_tokens(2, 256, cfg.vocab, seed=3, device=dev)
    tr_n, tr_r = LMTrainer(native, ddp=False), LMTrainer(ref, ddp=False)
    ln, lr_ = tr_n.loss(tok), tr_r.loss(tok)
    assert abs(ln.item() - lr_.item()) < 2e-3 * abs(lr_.item())
    ln.backward()
    lr_.backward()
    for (name, pn), (_, pr) in zip(native.named_parameters(), ref.named_parameters()):
        err = (pn.grad - pr.grad).abs().max().item() / max(pr.grad.abs().max().item(), 1e-6)
        assert err < 3e-2, (name, err)
    native.zero_grad(set_to_none=True)
    first = tr_n.step(tok).item()
    for _ in range(10):
        last = tr_n.step(tok).item()
    assert math.isfinite(last) and last < first
