"""CPU checks of the QAT step's host-side pieces."""

import torch
import torch.nn.functional as F


def test_linear_cross_entropy_matches_plain_path():
    from cdl_b200.train.qat import LinearCrossEntropy

    torch.manual_seed(0)
    h = torch.randn(300, 64, requires_grad=True)
    w = (0.05 * torch.randn(1000, 64)).requires_grad_()
    t = torch.randint(0, 1000, (300,))
    loss = LinearCrossEntropy.apply(h, w, t, 128)
    (2.0 * loss).backward()
    gh, gw = h.grad.clone(), w.grad.clone()
    h.grad = w.grad = None
    ref = F.cross_entropy(h @ w.t(), t)
    (2.0 * ref).backward()
    assert torch.allclose(loss, ref, rtol=1e-6)
    assert torch.allclose(gh, h.grad, rtol=1e-5, atol=1e-7)
    assert torch.allclose(gw, w.grad, rtol=1e-5, atol=1e-7)


def test_quantized_backward_backend_names():
    from cdl_b200.model.components.linear import QLinear

    q = QLinear(64, 32)
    for be in ("native", "nvfp4", "mxfp4", "mxfp8", "nvfp4_qbwd", "mxfp4_qbwd", "mxfp8_qbwd"):
        q.set_backend(be)
    try:
        q.set_backend("fp4")
    except ValueError:
        pass
    else:
        raise AssertionError("unknown backend accepted")


def test_cdl_quantizer_variants_build_with_their_optimizer_group():
    """cdl's quantizer variants in the QAT step: the classes apply_quant puts
    in each QLinear, and the extra AdamW group of the quantizers' own
    parameters at quant_lr (smollm2.py build_optimizer)."""
    import pytest

    from cdl_b200.model.components.linear import QLinear
    from cdl_b200.model.components.quant import ccdl, ecdl
    from cdl_b200.train import qat

    step = qat.QatStep(qat.SPECS["tiny"], torch.device("cpu"), backend="nvfp4", weight="nvfp4_ccdl",
                       activation="nvfp4_ecdl", quant_lr=1e-3)
    qls = [m for m in step.model.modules() if isinstance(m, QLinear)]
    assert len(qls) == step.n_quant == 14
    assert all(isinstance(m.weight_quant, ccdl.Nvfp4CascadedCdlQuantForWeight) for m in qls)
    assert all(isinstance(m.activation_quant, ecdl.Nvfp4ExtendedCdlQuantForActivation) for m in qls)
    assert step.optimizer == "torch"
    groups = step.opt.param_groups
    assert groups[-1]["lr"] == 1e-3 and len(groups[-1]["params"]) == 2 * 14  # log_q, log_alpha per weight
    assert not qls[0].activation_quant.log_kappa.requires_grad  # train_kappa=False
    with pytest.raises(ValueError):
        qat.QatStep(qat.SPECS["tiny"], torch.device("cpu"), weight="nvfp4_ccdl", optimizer="fused")
    with pytest.raises(ValueError):
        qat.apply_quant(torch.nn.Linear(4, 4), weight="fp3_cdl")


def test_lora_freeze_policy_and_lr_schedule():
    """cdl's parameter policy and LR factor: LoRA trains only the adapters
    (head untied and frozen); freeze_base trains the untied head; the plain
    untied run freezes only the input embedding; warmup + cosine factors."""
    import math

    from cdl_b200.train import qat

    spec, cpu = qat.SPECS["tiny"], torch.device("cpu")
    lora = qat.QatStep(spec, cpu, backend="nvfp4", use_lora=True, lora_r=4, lora_alpha=8)
    names = [n for n, p in lora.model.named_parameters() if p.requires_grad]
    assert len(names) == 2 * 14 and all(n.endswith((".lora.a", ".lora.b")) for n in names)
    assert lora.model.lm_head.weight is not lora.model.get_input_embeddings().weight
    fb = qat.QatStep(spec, cpu, backend="nvfp4", freeze_base=True)
    assert [n for n, p in fb.model.named_parameters() if p.requires_grad] == ["lm_head.weight"]
    un = qat.QatStep(spec, cpu, backend="nvfp4", untie=True)
    frozen = [n for n, p in un.model.named_parameters() if not p.requires_grad]
    assert frozen == ["model.embed_tokens.weight"]
    f = qat.lr_lambda(warmup_steps=4, lr_decay="cosine", max_steps=14, min_lr_ratio=0.1)
    assert [f(s) for s in range(4)] == [0.25, 0.5, 0.75, 1.0]
    assert f(4) == 1.0 and abs(f(9) - (0.1 + 0.45 * (1 + math.cos(math.pi * 0.5)))) < 1e-12 and f(20) == 0.1
    st = qat.QatStep(spec, cpu, backend="nvfp4", lr=1e-3, warmup_steps=10)
    assert st.opt.param_groups[0]["lr"] == 1e-4  # LambdaLR applies the first factor at construction


def test_evaluate_perplexity_on_cpu():
    """evaluate() = exp(token-weighted mean loss) over the batches, model left
    in its training mode (unquantized tiny model on the CPU)."""
    import math

    from cdl_b200.train import qat

    spec = qat.SPECS["tiny"]
    model = qat.build_model(spec, torch.device("cpu"), seed=0)
    batches = [torch.randint(0, spec.vocab, (2, 16), generator=torch.Generator().manual_seed(i)) for i in range(3)]
    model.train()
    ppl = qat.evaluate(model, batches, torch.device("cpu"))
    assert model.training
    with torch.no_grad():
        model.eval()
        mean = sum(float(qat.lm_loss(model, b)) for b in batches) / 3  # equal token counts per batch
    assert abs(ppl - math.exp(mean)) < 1e-6 * math.exp(mean) and abs(math.log(ppl) - math.log(spec.vocab)) < 0.5


def test_gradient_accumulation_matches_one_big_batch():
    """A list of micro-batches accumulates gradients before one optimizer
    step: the returned loss is their mean, and the update equals the step on
    the concatenated batch (equal token counts; unquantized model on CPU,
    fp32 gradients compared before the optimizer)."""
    from cdl_b200.train import qat

    spec, cpu = qat.SPECS["tiny"], torch.device("cpu")
    b1, b2 = (torch.randint(0, spec.vocab, (2, 16), generator=torch.Generator().manual_seed(i)) for i in (1, 2))
    a = qat.QatStep(spec, cpu, backend="none", lr=1e-3, seed=0)
    b = qat.QatStep(spec, cpu, backend="none", lr=1e-3, seed=0)
    for m in (a.model, b.model):
        m.float()
    grads = {}
    for name, st, ids in (("micro", a, [b1, b2]), ("whole", b, torch.cat([b1, b2]))):
        st.opt.step = lambda: None  # keep the parameters: compare the accumulated gradients
        st.opt.zero_grad = lambda set_to_none=True: None
        loss, _ = st.step(ids)
        grads[name] = (float(loss), [p.grad.clone() for p in st.params])
    assert abs(grads["micro"][0] - grads["whole"][0]) < 1e-5
    for x, y in zip(grads["micro"][1], grads["whole"][1]):
        assert torch.allclose(x, y, rtol=1e-4, atol=1e-6)


def test_fp32_master_weights_step():
    """fp32 master weights: the optimizer steps fp32 copies and writes them
    back into the bf16 parameters, which then equal the masters rounded."""
    from cdl_b200.train import qat

    spec, cpu = qat.SPECS["tiny"], torch.device("cpu")
    st = qat.QatStep(spec, cpu, backend="none", lr=1e-2, seed=0, fp32_master_weights=True)
    assert st.master_pairs and all(m.dtype == torch.float32 for _, m in st.master_pairs)
    p, m = st.master_pairs[3]
    before = p.detach().clone()
    ids = torch.randint(0, spec.vocab, (2, 16), generator=torch.Generator().manual_seed(0))
    st.step(ids)
    assert not torch.equal(p.detach(), before) and torch.equal(p.detach(), m.detach().to(p.dtype))
    assert all(q.grad is None for q in st.params)


def test_run_training_loop_checkpoints_and_resumes(tmp_path):
    """cdl's loop around the step: accumulation windows, max_steps, periodic
    checkpoint and evaluation, logging, then a resume from the checkpoint
    that continues the step count (unquantized tiny model on CPU)."""
    import numpy as np

    from cdl_b200.data import DeviceBlockLoader, build_from_tokens
    from cdl_b200.train import qat
    from cdl_b200.train.checkpoint import load_checkpoint

    spec, cpu = qat.SPECS["tiny"], torch.device("cpu")
    toks = np.random.default_rng(0).integers(0, spec.vocab, 32 * 20)
    cache = build_from_tokens(tmp_path / "cache", toks, seq_len=32, num_test_blocks=4)
    train = DeviceBlockLoader(cache.train_dataset, 2, "cpu")
    test = DeviceBlockLoader(cache.test_dataset, 2, "cpu", shuffle=False)
    logs = []
    st = qat.QatStep(spec, cpu, backend="none", lr=1e-3, seed=0, warmup_steps=2)
    gs = qat.run_training(st, train, grad_accum_steps=2, max_steps=3, test_batches=test, eval_every=2,
                          save_every=2, checkpoint_path=tmp_path / "last.ckpt", log_every=1,
                          log=lambda *a: logs.append(a))
    assert gs == 3
    train_logs = [a for a in logs if a[1] is not None]
    evals = [a for a in logs if a[1] is None]
    assert [a[0] for a in train_logs] == [1, 2, 3] and [a[0] for a in evals] == [2, 3]
    assert all(1.0 < a[3] < 2 * spec.vocab for a in evals)  # perplexities
    ck = torch.load(tmp_path / "last.ckpt", weights_only=False)
    assert ck["global_step"] == 3 and ck["lr_scheduler"]["last_epoch"] == 3

    st2 = qat.QatStep(spec, cpu, backend="none", lr=1e-3, seed=1, warmup_steps=2)
    _, start = load_checkpoint(tmp_path, st2.model, st2.opt, st2.lr_scheduler, cpu)
    assert start == 3
    for a, b in zip(st.model.parameters(), st2.model.parameters()):
        assert torch.equal(a.detach(), b.detach())
    # 8 batches = 4 steps per epoch: the resumed run ends its first epoch at step 4
    assert qat.run_training(st2, train, grad_accum_steps=2, start_step=start, max_steps=10) == 4
    assert qat.run_training(st2, train, epochs=2, grad_accum_steps=2, start_step=4, max_steps=6) == 6


def test_amax_arena_hands_out_zeroed_words_within_a_step():
    """The fused kernels' amax words: inside a step, consecutive slices of one
    buffer zeroed when the step begins; outside a step, or once the buffer is
    used up, fresh zero-filled tensors."""
    from cdl_b200 import _lib
    from cdl_b200.model.components import fused

    dev = torch.device("cpu")
    outside = fused.new_amax(dev)
    assert outside.shape == (_lib.AMAX_WORDS,) and not outside.any()
    fused.begin_step(dev)
    try:
        a, b = fused.new_amax(dev), fused.new_amax(dev, 2)
        assert a.shape == (_lib.AMAX_WORDS,) and b.shape == (2, _lib.AMAX_WORDS)
        assert a.data_ptr() != b.data_ptr() and not a.any() and not b.any()
        a.fill_(7)  # a kernel writes its word
        assert not b.any()
        rest = fused._ARENA.SLOTS - fused._ARENA.used
        fused.new_amax(dev, rest)  # the last slots
        spill = fused.new_amax(dev)  # beyond the buffer: a fresh tensor
        assert not spill.any() and spill.data_ptr() != a.data_ptr()
    finally:
        fused.end_step()
    fused.begin_step(dev)  # the next step zeroes the words again
    try:
        assert not fused.new_amax(dev).any()
    finally:
        fused.end_step()
    assert not fused._ARENA.active


def test_dgrad_sum_bookkeeping():
    """Linears that read one encoded input join one sum: the users are
    counted in the forward; a new sum starts once a backward has begun."""
    from cdl_b200.core.mm import blockscaled

    codes = torch.zeros(4, dtype=torch.uint8)
    s1 = blockscaled._join_dgrad_sum(codes)
    s2 = blockscaled._join_dgrad_sum(codes)
    assert s1 is s2 and s1.users == 2 and s1.done == 0
    s1.done = 1  # the backward of one of them ran
    s3 = blockscaled._join_dgrad_sum(codes)
    assert s3 is not s1 and s3.users == 1
