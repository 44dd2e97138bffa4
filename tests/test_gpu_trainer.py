"""KernelOptGRPOTrainer._get_per_token_logps_and_entropies (reference
python/kernel_opt/trainer.py:38-131) driven without trl: a stand-in `trl` module provides a
GRPOTrainer base class with only what the override uses, and a tiny causal LM supplies the
logits.  The override's result (one K1 launch per chunk on the strided completion window)
must equal the eager computation TRL does (slice, temperature, log_softmax, entropy), and
its gradient must reach the model."""
import sys
import types

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


class _TinyLM(torch.nn.Module):
    def __init__(self, vocab=3000, hidden=64):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.emb = torch.nn.Parameter(torch.randn(vocab, hidden, generator=g) * 0.5)
        self.head = torch.nn.Parameter(torch.randn(hidden, vocab, generator=g) * 0.5)

    def forward(self, input_ids, attention_mask=None, logits_to_keep=None, use_cache=False):
        h = self.emb[input_ids].cumsum(1) / torch.arange(1, input_ids.shape[1] + 1,
                                                         device=input_ids.device)[:, None]
        if logits_to_keep:
            h = h[:, -logits_to_keep:]
        return types.SimpleNamespace(logits=(h @ self.head).to(torch.bfloat16))


@pytest.fixture()
def trainer_cls(monkeypatch):
    class GRPOTrainer:  # the stand-in base class
        def _get_per_token_logps_and_entropies(self, *a, **k):
            raise AssertionError("parent called")

    fake = types.ModuleType("trl")
    fake.GRPOTrainer = GRPOTrainer
    monkeypatch.setitem(sys.modules, "trl", fake)
    sys.modules.pop("kernel_opt.trainer", None)
    import kernel_opt
    cls = kernel_opt.KernelOptGRPOTrainer
    yield cls
    sys.modules.pop("kernel_opt.trainer", None)


def _eager(model, input_ids, attention_mask, logits_to_keep, temperature):
    logits = model(input_ids, attention_mask, logits_to_keep=logits_to_keep + 1).logits
    logits = logits[:, :-1, :][:, -logits_to_keep:, :].clone()
    logits = logits.div_(temperature).float()  # bf16 in-place division, as TRL does
    ids = input_ids[:, -logits_to_keep:]
    logp_all = F.log_softmax(logits, -1)
    logps = logp_all.gather(-1, ids.unsqueeze(-1)).squeeze(-1)
    ent = -(logp_all.exp() * logp_all).sum(-1)
    return logps, ent


@pytest.mark.parametrize("batch_size", [None, 2])
@pytest.mark.parametrize("inplace", [False, True])
def test_override_matches_eager_and_backprops(trainer_cls, batch_size, inplace):
    model = _TinyLM().cuda()
    tr = trainer_cls(k1_inplace_backward=inplace)
    tr.temperature = 0.7
    tr.model_kwarg_keys = {"input_ids", "attention_mask", "logits_to_keep", "use_cache"}
    g = torch.Generator().manual_seed(1)
    input_ids = torch.randint(0, 3000, (5, 40), generator=g).cuda()
    mask = torch.ones_like(input_ids)
    K = 17
    logps, ents = tr._get_per_token_logps_and_entropies(model, input_ids, mask, K,
                                                        batch_size=batch_size,
                                                        compute_entropy=True)
    ref_lp, ref_ent = _eager(model, input_ids, mask, K, tr.temperature)
    assert logps.shape == (5, K) and ents.shape == (5, K)
    assert not ents.requires_grad and logps.requires_grad
    torch.testing.assert_close(logps, ref_lp, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(ents, ref_ent, rtol=1e-4, atol=1e-5)
    logps.sum().backward()
    grad_ours = model.head.grad.clone()
    model.zero_grad()
    ref_lp.sum().backward()
    torch.testing.assert_close(grad_ours, model.head.grad, rtol=2e-2, atol=2e-3)


def test_override_equals_reference_sequence_bitwise(trainer_cls):
    """The override's logps and the logits gradient equal what the reference's own
    sequence (slice, in-place div_ by the temperature, K1) gives with our K1, bit for bit."""
    import kernel_opt
    from kernel_opt import grpo

    model = _TinyLM().cuda()
    tr = trainer_cls()
    tr.temperature = 0.9
    tr.model_kwarg_keys = {"input_ids", "attention_mask", "logits_to_keep", "use_cache"}
    input_ids = torch.randint(0, 3000, (4, 30), generator=torch.Generator().manual_seed(3)).cuda()
    K = 12
    captured = {}
    fwd = model.forward

    def spy(*a, **k):
        out = fwd(*a, **k)
        out.logits.retain_grad()
        captured["logits"] = out.logits
        return out

    model.forward = spy
    logps, _ = tr._get_per_token_logps_and_entropies(model, input_ids, torch.ones_like(input_ids), K)
    logps.sum().backward()
    g_ours = captured["logits"].grad.clone()

    x0 = fwd(input_ids, None, logits_to_keep=K + 1).logits
    x0.retain_grad()
    logits = x0 * 1  # the in-place division below must not touch x0 (its .grad is compared)
    w = grpo.completion_window(logits, K)
    w.div_(tr.temperature)
    ref, _, _ = kernel_opt.fused_logprob_entropy(w, input_ids[:, -K:].contiguous())
    ref.sum().backward()
    torch.testing.assert_close(logps.detach(), ref.detach(), rtol=0, atol=0)
    torch.testing.assert_close(g_ours, x0.grad, rtol=0, atol=0)


def test_multimodal_falls_back_to_parent(trainer_cls):
    tr = trainer_cls()
    with pytest.raises(AssertionError, match="parent called"):
        tr._get_per_token_logps_and_entropies(None, None, None, 3, pixel_values=object())


class _TinyDecoder(torch.nn.Module):
    def __init__(self, vocab, hidden):
        super().__init__()
        g = torch.Generator().manual_seed(5)
        self.emb = torch.nn.Parameter((torch.randn(vocab, hidden, generator=g) * 0.5))

    def forward(self, input_ids, attention_mask=None, use_cache=False):
        h = self.emb[input_ids].cumsum(1) / torch.arange(1, input_ids.shape[1] + 1,
                                                         device=input_ids.device)[:, None]
        return (h.to(torch.bfloat16),)


class _TinyHFLM(torch.nn.Module):
    """Shaped like a transformers causal LM: decoder + bias-free lm_head."""

    def __init__(self, vocab=3000, hidden=64):
        super().__init__()
        self.decoder = _TinyDecoder(vocab, hidden)
        self.lm_head = torch.nn.Linear(hidden, vocab, bias=False).to(torch.bfloat16)
        self.config = types.SimpleNamespace()

    def get_decoder(self):
        return self.decoder

    def get_output_embeddings(self):
        return self.lm_head

    def forward(self, input_ids, attention_mask=None, logits_to_keep=None, use_cache=False):
        h = self.decoder(input_ids, attention_mask)[0]
        if logits_to_keep:
            h = h[:, -logits_to_keep:]
        return types.SimpleNamespace(logits=self.lm_head(h))


@pytest.mark.parametrize("batch_size", [None, 2])
def test_fused_lm_head_option(trainer_cls, batch_size):
    model = _TinyHFLM().cuda()
    input_ids = torch.randint(0, 3000, (5, 40), generator=torch.Generator().manual_seed(6)).cuda()
    mask = torch.ones_like(input_ids)
    K = 17
    res = {}
    for fused in (False, True):
        tr = trainer_cls(k1_fused_lm_head=fused)
        tr.temperature = 0.7
        tr.model_kwarg_keys = {"input_ids", "attention_mask", "logits_to_keep", "use_cache"}
        model.zero_grad()
        lp, ent = tr._get_per_token_logps_and_entropies(model, input_ids, mask, K,
                                                        batch_size=batch_size,
                                                        compute_entropy=True)
        (lp * torch.linspace(-1, 1, K, device="cuda")).sum().backward()
        res[fused] = (lp.detach(), ent, model.lm_head.weight.grad.clone(),
                      model.decoder.emb.grad.clone())
    a, b = res[False], res[True]
    torch.testing.assert_close(b[0], a[0], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(b[1], a[1], rtol=1e-4, atol=1e-5)
    for ga, gb in zip(a[2:], b[2:]):
        torch.testing.assert_close(gb.float(), ga.float(), rtol=2e-2,
                                   atol=2e-3 * float(ga.float().abs().max()))


def test_fused_lm_head_falls_back_for_soft_capped_models(trainer_cls):
    model = _TinyHFLM().cuda()
    model.config.final_logit_softcapping = 30.0
    tr = trainer_cls(k1_fused_lm_head=True)
    tr.temperature = 1.0
    tr.model_kwarg_keys = {"input_ids", "attention_mask", "logits_to_keep", "use_cache"}
    ids = torch.randint(0, 3000, (2, 12), generator=torch.Generator().manual_seed(7)).cuda()
    with pytest.warns(UserWarning, match="k1_fused_lm_head"):
        lp, _ = tr._get_per_token_logps_and_entropies(model, ids, torch.ones_like(ids), 5)
    assert lp.shape == (2, 5)
