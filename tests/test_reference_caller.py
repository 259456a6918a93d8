"""The reference's own caller drives the drop-in classes (CPU, kernels faked by the oracle).

``Qwen3Attention.forward`` (src/nanovllm_ascend/models/qwen3.py:70-119 in
Pla-Yer/nano_vllm_ascend) is imported from a reference checkout -- the
directory named by $NVK_REFERENCE, else a ``reference`` checkout beside this
repository -- and is skipped when none is present (the GPU box has none).
``torch_npu`` is stubbed as the reference's own tests stub it
(tests/test_decode_graph.py:11-87 there): ``npu_rms_norm`` and
``npu_rotary_mul`` become fp32 torch restatements, and the NPU attention
classes of ``nanovllm_ascend.layers`` are replaced by this package's
``PagedAttention`` / ``BatchPrefillAttention``, exactly the import swap a
maintainer makes. The pool is this package's ``PagedKVCache`` and the
metadata its ``BlockManager``'s.

The device kernels are replaced by the CPU oracle (``ops`` functions patched),
so what this checks is the host contract: the reference calls every drop-in
with its own keyword arguments and order (write -> get_physical_cache ->
attention), prefill (dense, then paged with a prefix-cache hit) and decode
steps produce the oracle's pool bit for bit and its attention within the
attention tolerance, and the same layers run inside ``DecodeGraphRunner``
(with a stand-in graph backend) through the fused-append path.
"""

from __future__ import annotations

import contextlib
import importlib
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import nano_vllm_ascend_b200 as nvk
from nano_vllm_ascend_b200 import ops
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits

D, H, KVH, HIDDEN, BS = 128, 16, 8, 256, 16


def reference_src() -> Path | None:
    cands = [os.environ.get("NVK_REFERENCE", ""), str(Path(__file__).resolve().parents[2] / "reference")]
    for c in cands:
        if c and (Path(c) / "src" / "nanovllm_ascend" / "models" / "qwen3.py").exists():
            return Path(c) / "src"
    return None


def _rms_norm(x, weight, epsilon=1e-6):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + epsilon) * weight.float()
    return y.to(x.dtype), None


def _rotary_mul(x, cos, sin, rotary_mode="half"):
    assert rotary_mode == "half"
    xf = x.float()
    half = xf.shape[-1] // 2
    rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
    return (xf * cos.float() + rot * sin.float()).to(x.dtype)


def _np(t: torch.Tensor) -> np.ndarray:
    """Shared-memory uint16 view of a CPU bf16 tensor (writes land in the tensor)."""
    return t.view(torch.int16).numpy().view(np.uint16)


class OracleKernels:
    """Stands in for the CUDA entry points with the oracle, on CPU tensors."""

    def __init__(self):
        self.calls = []

    def kv_append(self, kc, vc, k, v, slots, error_word=None):
        self.calls.append("append")
        orc.kv_append(_np(kc), _np(vc), bits(k), bits(v), slots.numpy())

    def paged_decode(self, out, q, kc, vc, tables, ctx, scale, ws, num_ctas=0, new_key=None, new_value=None,
                     slot_mapping=None):
        self.calls.append("decode+append" if slot_mapping is not None else "decode")
        if slot_mapping is not None:
            orc.kv_append(_np(kc), _np(vc), bits(new_key), bits(new_value), slot_mapping.numpy())
        res = orc.paged_decode(bits(q), _np(kc), _np(vc), tables.numpy(), ctx.numpy(), scale)
        out.copy_(torch.from_numpy(res).to(torch.bfloat16))
        return out

    def paged_prefill(self, out, q, kc, vc, tables, cu_q, kv_lens, max_q_len, scale, error_word=None):
        self.calls.append("paged_prefill")
        res = orc.paged_prefill(bits(q), _np(kc), _np(vc), tables.numpy(), cu_q.numpy(), kv_lens.numpy(), scale)
        out.copy_(torch.from_numpy(res).to(torch.bfloat16))
        return out

    def dense_prefill(self, out, q, k, v, cu_q, cu_kv, max_q_len, scale, error_word=None):
        self.calls.append("dense_prefill")
        res = orc.dense_prefill(bits(q), bits(k), bits(v), cu_q.numpy(), cu_kv.numpy(), scale)
        out.copy_(torch.from_numpy(res).to(torch.bfloat16))
        return out


class NoErrors:
    word = None

    def raise_if_flagged(self):
        pass

    def launched(self, *names):
        pass

    def watch(self, name, word):
        return name


@pytest.fixture
def reference(monkeypatch):
    src = reference_src()
    if src is None:
        pytest.skip("no reference checkout (set NVK_REFERENCE)")
    fake_npu = types.ModuleType("torch_npu")
    fake_npu.npu_rms_norm = _rms_norm
    fake_npu.npu_rotary_mul = _rotary_mul
    monkeypatch.setitem(sys.modules, "torch_npu", fake_npu)
    monkeypatch.syspath_prepend(str(src))
    for name in [m for m in sys.modules if m == "nanovllm_ascend" or m.startswith("nanovllm_ascend.")]:
        monkeypatch.delitem(sys.modules, name)
    layers = importlib.import_module("nanovllm_ascend.layers")
    # the maintainer's swap: the NPU attention classes become the drop-ins
    monkeypatch.setattr(layers, "NpuPagedAttention", nvk.NpuPagedAttention, raising=False)
    monkeypatch.setattr(layers, "NpuBatchPrefillAttention", nvk.NpuBatchPrefillAttention, raising=False)
    qwen3 = importlib.import_module("nanovllm_ascend.models.qwen3")
    rope_mod = importlib.import_module("nanovllm_ascend.layers.rotary_embedding")
    # device work on CPU: the oracle replaces the kernels
    kernels = OracleKernels()
    for name in ("kv_append", "paged_decode", "paged_prefill", "dense_prefill"):
        monkeypatch.setattr(ops, name, getattr(kernels, name))
    monkeypatch.setattr(torch.cuda, "device", lambda *_: contextlib.nullcontext())
    monkeypatch.setattr(nvk.device_errors, "state", lambda *_: NoErrors())
    monkeypatch.setattr(nvk.PagedAttention, "workspace_bytes", lambda self, b: 64)
    monkeypatch.setattr(importlib.import_module("nano_vllm_ascend_b200.paged_attention"), "shared_workspace",
                        lambda device, nbytes, shape=(): torch.zeros(nbytes, dtype=torch.uint8))
    grad = torch.is_grad_enabled()
    torch.set_grad_enabled(False)  # the reference's runner works under torch.inference_mode()
    yield SimpleNamespace(qwen3=qwen3, rope=rope_mod, kernels=kernels)
    torch.set_grad_enabled(grad)
    for name in [m for m in sys.modules if m == "nanovllm_ascend" or m.startswith("nanovllm_ascend.")]:
        sys.modules.pop(name, None)


def make_layers(ref, n_layers, seed=0):
    config = SimpleNamespace(hidden_size=HIDDEN, num_attention_heads=H, num_key_value_heads=KVH, head_dim=D,
                             rms_norm_eps=1e-6, attention_bias=False, nanovllm_block_size=BS,
                             nanovllm_max_model_len=1024)
    g = torch.Generator().manual_seed(seed)
    layers = []
    for i in range(n_layers):
        layer = ref.qwen3.Qwen3Attention(config, layer_idx=i)
        for p in layer.parameters():
            p.data = (torch.randn(p.shape, generator=g) * (0.05 if p.dim() == 2 else 1.0) + (0 if p.dim() == 2 else 1)
                      ).to(torch.bfloat16)
        layers.append(layer)
    assert isinstance(layers[0].paged_attn, nvk.PagedAttention)
    assert isinstance(layers[0].prefill_attn, nvk.BatchPrefillAttention)
    return config, layers


def expected_layer(layer, hidden, cos, sin, kc, vc, md, is_prefill):
    """The same layer restated without the drop-ins: projections and the stubbed
    norm / rotary as in qwen3.py:79-89, then the oracle's append and attention."""
    t = hidden.shape[0]
    q = F.linear(hidden, layer.q_proj.weight).view(t, H, D)
    k = F.linear(hidden, layer.k_proj.weight).view(t, KVH, D)
    v = F.linear(hidden, layer.v_proj.weight).view(t, KVH, D)
    q = _rms_norm(q, layer.q_norm.weight, 1e-6)[0]
    k = _rms_norm(k, layer.k_norm.weight, 1e-6)[0]
    c = cos.to(q.dtype).view(t, 1, D)
    s = sin.to(q.dtype).view(t, 1, D)
    q, k = _rotary_mul(q, c, s), _rotary_mul(k, c, s)
    orc.kv_append(kc, vc, bits(k), bits(v), md.slot_mapping.numpy())
    if is_prefill and md.use_paged_prefill:
        cu = np.array([0] + list(md.actual_seq_lengths_q))
        att = orc.paged_prefill(bits(q), kc, vc, md.block_tables.numpy(), cu, md.context_lens.numpy(), D ** -0.5)
    elif is_prefill:
        cu = np.array([0] + list(md.actual_seq_lengths_q))
        cukv = np.array([0] + list(md.actual_seq_lengths_kv))
        att = orc.dense_prefill(bits(q), bits(k), bits(v), cu, cukv, D ** -0.5)
    else:
        att = orc.paged_decode(bits(q), kc, vc, md.block_tables.numpy(), md.context_lens.numpy(), D ** -0.5)
    att = torch.from_numpy(att).to(torch.bfloat16)
    return F.linear(att.reshape(t, H * D), layer.o_proj.weight)


def run_and_check(ref, layers, kv, pool, hidden, positions, md, is_prefill, what):
    rope = ref.rope.RotaryEmbedding(D, max_position_embeddings=1024)
    cos, sin = rope(positions.view(1, -1))
    cos, sin = cos.view(-1, D), sin.view(-1, D)
    for layer in layers:
        got = layer(hidden, (cos, sin), kv, md, is_prefill)
        kc, vc = pool[0][layer.layer_idx], pool[1][layer.layer_idx]
        want = expected_layer(layer, hidden, cos, sin, kc, vc, md, is_prefill)
        assert np.array_equal(bits(kv.key_cache[layer.layer_idx]), kc), f"{what}: key pool"
        assert np.array_equal(bits(kv.value_cache[layer.layer_idx]), vc), f"{what}: value pool"
        assert_close(got.float().numpy(), want.float().numpy(), f"{what} layer {layer.layer_idx}")


def test_reference_qwen3_attention_drives_the_drop_ins(reference):
    ref = reference
    n_layers, nb = 2, 48
    _, layers = make_layers(ref, n_layers)
    bm = nvk.BlockManager(nb, BS, "cpu")
    kv = nvk.PagedKVCache(n_layers, nb, BS, KVH, D, torch.bfloat16, "cpu")
    kv.key_cache.zero_()
    kv.value_cache.zero_()
    pool = (bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
    g = torch.Generator().manual_seed(1)
    prompt_a = torch.randint(0, 1000, (70,), generator=g)
    # request 0: dense prefill of 70 tokens, then its 4 full blocks are cached
    md = bm.prepare_prefill_metadata([0], [70], [0], [[]])
    assert not md.use_paged_prefill
    hidden = (torch.randn(70, HIDDEN, generator=g)).to(torch.bfloat16)
    run_and_check(ref, layers, kv, pool, hidden, torch.arange(70), md, True, "dense prefill")
    bm.cache_full_blocks(slot=0, token_ids=prompt_a, num_cached_blocks=0, num_full_blocks=70 // BS)
    # request 1 shares 64 tokens (4 blocks): prefix hit, paged prefill of its 30-token suffix
    prompt_b = torch.cat([prompt_a[:64], torch.randint(0, 1000, (30,), generator=g)])
    hit = bm.find_longest_prefix_blocks(prompt_b, max_cache_blocks=94 // BS)
    assert len(hit) == 4
    md = bm.prepare_prefill_metadata([1], [30], [64], [hit])
    assert md.use_paged_prefill
    hidden = (torch.randn(30, HIDDEN, generator=g)).to(torch.bfloat16)
    run_and_check(ref, layers, kv, pool, hidden, torch.arange(64, 94), md, True, "paged prefill (prefix hit)")
    # three decode steps of both sequences (the first crosses a block boundary for request 1)
    lens = [70, 94]
    for step in range(3):
        md = bm.prepare_decode_metadata([0, 1], lens, q_len=1)
        hidden = (torch.randn(2, HIDDEN, generator=g)).to(torch.bfloat16)
        run_and_check(ref, layers, kv, pool, hidden, torch.tensor(lens), md, False, f"decode step {step}")
        lens = [n + 1 for n in lens]
    assert ref.kernels.calls.count("dense_prefill") == n_layers
    assert ref.kernels.calls.count("paged_prefill") == n_layers
    assert ref.kernels.calls.count("decode") == 3 * n_layers


class GraphModel:
    """Qwen3ForCausalLM's decode contract (qwen3.py:203-221) over the reference's
    attention layers: embedding rows in, the last layer's output as logits."""

    def __init__(self, ref, layers, embed):
        self.layers, self.embed = layers, embed
        self.rope = ref.rope.RotaryEmbedding(D, max_position_embeddings=1024)

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill=False):
        hidden = self.embed[input_ids_flat]
        cos, sin = self.rope(position_ids_flat.view(1, -1))
        pe = (cos.view(-1, D), sin.view(-1, D))
        for layer in self.layers:
            hidden = layer(hidden, pe, kv_cache, attn_metadata, is_prefill)
        return SimpleNamespace(logits=hidden)


def test_reference_layers_inside_the_decode_graph_runner_use_the_fused_append(reference):
    from tests.test_graph_runner import FakeBackend

    ref = reference
    n_layers, nb = 2, 32
    _, layers = make_layers(ref, n_layers, seed=5)
    g = torch.Generator().manual_seed(6)
    embed = (torch.randn(100, HIDDEN, generator=g)).to(torch.bfloat16)
    bm = nvk.BlockManager(nb, BS, "cpu")
    kv = nvk.PagedKVCache(n_layers, nb, BS, KVH, D, torch.bfloat16, "cpu")
    kv.key_cache.copy_(torch.randn(kv.key_cache.shape, generator=g).to(torch.bfloat16))
    kv.value_cache.copy_(torch.randn(kv.value_cache.shape, generator=g).to(torch.bfloat16))
    lens = [40, 17, 33]
    bm.prepare_prefill_metadata([0, 1, 2], lens, [0, 0, 0], [[], [], []])
    runner = nvk.DecodeGraphRunner(GraphModel(ref, layers, embed), kv, batch_sizes=[3], max_model_len=256,
                                   block_size=BS, device="cpu", backend=FakeBackend())
    pool = (bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
    ids = torch.tensor([3, 50, 7])
    md = bm.prepare_decode_metadata([0, 1, 2], lens, q_len=1)
    logits = runner.forward(ids, torch.tensor(lens), md)
    assert logits is not None and runner.stats_dict()["captures"] == 1
    # warm-up and capture both ran the layers with the append fused into decode
    assert ref.kernels.calls.count("decode+append") == 2 * n_layers
    assert "append" not in ref.kernels.calls
    # the stand-in backend does not replay: the slot's logits are the capture run's; the
    # pool holds this step's rows exactly once per slot (the warm-up rewrote the same rows)
    rope = ref.rope.RotaryEmbedding(D, max_position_embeddings=1024)
    cos, sin = rope(torch.tensor(lens).view(1, -1))
    hidden = embed[ids]
    md_static = runner.slot(3).metadata(md)
    for layer in layers:
        kc, vc = pool[0][layer.layer_idx], pool[1][layer.layer_idx]
        hidden = expected_layer(layer, hidden, cos.view(-1, D), sin.view(-1, D), kc, vc, md_static, False)
        assert np.array_equal(bits(kv.key_cache[layer.layer_idx]), kc)
    assert_close(logits.float().numpy(), hidden.float().numpy(), "graph runner logits")
