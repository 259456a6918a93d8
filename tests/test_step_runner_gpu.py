"""StepRunner (the ModelRunner step drivers on the device path) against a
plain-torch restatement of the same Qwen3-shaped model.

A small model (2 layers, hidden 256, Qwen3-0.6B attention shapes, vocabulary
512) serves sequences shaped like the reference's EngineCore traffic
(src/nanovllm_ascend/engine.py:26-51 in Pla-Yer/nano_vllm_ascend): prefills
(one hitting another's cached prefix), decode steps at batch sizes with a
graph (4, 2) and without one (3, eager), a sequence freed and its row reused.
The reference recomputes every live sequence from scratch each step with
fp32 causal attention over its own K/V, fed the runner's own tokens (teacher
forcing), and checks that

* every token the runner picked is a greedy choice of the reference logits
  (its logit within 0.05 of the maximum: the kernels' bf16 rounding may
  reorder near-ties),
* every K/V row the runner wrote into the pool (layer 0 and the last layer,
  through the block manager's tables) matches the reference's: layer 0's
  within the attention tolerance; the last layer's, which inherit one layer
  of bf16 rounding differences through attention, projections and MLP,
  within two bf16 ulps at magnitude 8 (0.125) plus 2e-2 relative.
"""

from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

from nano_vllm_ascend_b200.step_runner import ModelShape, StepRunner, StepSequence, _rms_norm

pytestmark = pytest.mark.gpu

SHAPE = ModelShape(num_layers=2, hidden_size=256, num_heads=16, num_kv_heads=8, head_dim=128,
                   intermediate_size=512, vocab_size=512, max_position=4096)
ATOL, RTOL, LOGIT_TOL = 2e-2, 1e-2, 5e-2
DEEP_ATOL, DEEP_RTOL = 0.125, 2e-2  # rows of layers behind at least one attention layer


def Seq(seq_id, prompt):
    return StepSequence(seq_id, prompt, sampling_params=SimpleNamespace(temperature=0.0))


def _head_norm_rope(x, w, cos, sin, eps):
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16).float()
    half = y.shape[-1] // 2
    rot = torch.cat([-y[..., half:], y[..., :half]], dim=-1)
    c = cos.to(torch.bfloat16).float()[:, None]
    s = sin.to(torch.bfloat16).float()[:, None]
    return (y * c + rot * s).to(torch.bfloat16)


def reference_forward(model, tokens):
    """Logits of the last position and each layer's rotated K and V rows, in plain torch."""
    s = model.shape
    ids = tokens.to(model.embed.device)
    n = ids.numel()
    pos = torch.arange(n, device=ids.device)
    cos, sin = model.cos[pos], model.sin[pos]
    x = model.embed[ids]
    kv = []
    g = s.num_heads // s.num_kv_heads
    causal = torch.ones(n, n, dtype=torch.bool, device=ids.device).tril()
    for layer in model.layers:
        h = _rms_norm(x, layer.in_norm, s.rms_norm_eps)
        qkv = F.linear(h, layer.qkv).view(n, -1, s.head_dim)
        q = _head_norm_rope(qkv[:, :s.num_heads], layer.q_norm, cos, sin, s.rms_norm_eps)
        k = _head_norm_rope(qkv[:, s.num_heads:s.num_heads + s.num_kv_heads], layer.k_norm, cos, sin,
                            s.rms_norm_eps)
        v = qkv[:, s.num_heads + s.num_kv_heads:]
        kv.append((k, v))
        qg = q.float().view(n, s.num_kv_heads, g, s.head_dim)
        sc = torch.einsum("tkgd,nkd->kgtn", qg, k.float()) * s.head_dim ** -0.5
        p = torch.softmax(sc.masked_fill(~causal, float("-inf")), dim=-1)
        attn = torch.einsum("kgtn,nkd->tkgd", p, v.float()).reshape(n, -1).to(torch.bfloat16)
        x = x + F.linear(attn, layer.o)
        h = _rms_norm(x, layer.post_norm, s.rms_norm_eps)
        gate, up = F.linear(h, layer.gate_up).chunk(2, dim=-1)
        x = x + F.linear(F.silu(gate) * up, layer.down)
    h = _rms_norm(x, model.final_norm, s.rms_norm_eps)
    return h[-1].float() @ model.embed.float().T, kv


def check_sequences(runner, seqs, what):
    bm = runner.block_manager
    for seq in seqs:
        tokens = seq.token_ids()
        logits, kv = reference_forward(runner.model, tokens)
        # the runner's next token is a greedy choice of the reference's logits
        tok = seq.next_token_id
        assert float(logits[tok]) >= float(logits.max()) - LOGIT_TOL, \
            f"{what}: seq {seq.seq_id} picked {tok} ({float(logits[tok]):.4f}) vs max {float(logits.max()):.4f}"
        # the pool holds the reference's K/V rows at the sequence's slots
        row = runner._rows[seq.seq_id]
        table = torch.tensor(bm.block_tables[row], dtype=torch.int64, device=runner.device)
        n = tokens.numel()
        slots = table[torch.arange(n, device=runner.device) // bm.block_size] * bm.block_size \
            + torch.arange(n, device=runner.device) % bm.block_size
        for layer in (0, len(runner.model.layers) - 1):
            k_ref, v_ref = kv[layer]
            kc, vc = runner.kv_cache.get_physical_cache(layer)
            k_got = kc.reshape(-1, *kc.shape[2:])[slots].float()
            v_got = vc.reshape(-1, *vc.shape[2:])[slots].float()
            atol, rtol = (ATOL, RTOL) if layer == 0 else (DEEP_ATOL, DEEP_RTOL)
            for got, want, name in ((k_got, k_ref.float(), "K"), (v_got, v_ref.float(), "V")):
                err = (got - want).abs()
                assert bool((err <= atol + rtol * want.abs()).all()), \
                    f"{what}: seq {seq.seq_id} layer {layer} {name} rows off by up to {float(err.max())}"


def test_step_runner_prefill_and_decode_match_the_reference_model(cuda_device):
    runner = StepRunner(SHAPE, cuda_device, max_model_len=1024, num_blocks=64, block_size=128, max_num_seqs=8,
                        enable_prefix_cache=True, decode_graph_batch_sizes=[1, 2, 4], seed=3)
    g = torch.Generator().manual_seed(11)
    try:
        a = Seq(10, torch.randint(0, 512, (300,), generator=g))
        b = Seq(11, torch.randint(0, 512, (129,), generator=g))
        c = Seq(12, torch.randint(0, 512, (60,), generator=g))
        runner.prepare_sequences([a, b, c])
        runner.prefill([a, b, c])
        check_sequences(runner, [a, b, c], "prefill")
        # d shares a's first two blocks: a prefix-cache hit, paged prefill of its suffix
        d = Seq(13, torch.cat([a.prompt_token_ids[:256], torch.randint(0, 512, (40,), generator=g)]))
        runner.prepare_sequences([d])
        assert d.cached_prefix_len == 256
        runner.prefill([d])
        check_sequences(runner, [d], "prefill (prefix hit)")
        for step in range(3):  # batch 4: captured, then replayed
            runner.decode([a, b, c, d])
            check_sequences(runner, [a, b, c, d], f"decode bs4 step {step}")
        runner.free_seq(c)
        for step in range(2):  # batch 3: no graph, eager
            runner.decode([a, b, d])
            check_sequences(runner, [a, b, d], f"decode bs3 step {step}")
        e = Seq(14, torch.randint(0, 512, (5,), generator=g))  # reuses c's row
        runner.prepare_sequences([e])
        runner.prefill([e])
        for step in range(2):  # batch 2: captured, then replayed
            runner.decode([e, b])
            check_sequences(runner, [e, b], f"decode bs2 step {step}")
        stats = runner.decode_graph_stats()
        assert stats["captures"] == 2 and stats["replays"] == 5 and stats["fallbacks"] == 2
    finally:
        runner.release()
