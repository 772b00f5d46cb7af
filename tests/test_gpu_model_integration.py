"""The drop-in on a real decoder: a small randomly initialised Qwen2 model
(transformers' own modules: embeddings, projections with bias, RMSNorm, MLP,
rotary embedding) runs its attention layers through this package --
``rope_append`` into preallocated layer caches, ``flex_attention_forward``
on the step's tile plan, ``lm_head_argmax`` for the next tokens -- and is
compared with the same weights run the reference's way: transformers'
``apply_rotary_pos_emb``, softmax attention over the dense 0/-inf mask in
fp32, ``F.linear`` + ``argmax`` (D:337-351, D:72-135, D:1057-1064).

Two steps: a packed prefill of three prompts (block-diagonal causal), then a
verification step whose rows (new chunks of each block) attend to their
block's cached prompt rows and causally to each other.  Ids must agree on at
least 97 % of rows; the others must be near-ties of the reference logits
(bf16 attention against fp32).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HQ, HKV, D, HID, LAYERS, VOCAB = 4, 2, 128, 512, 2, 2048


@pytest.fixture(scope="module")
def model():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Config, Qwen2ForCausalLM

    from hsd_b200 import _native
    _native.load()
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=VOCAB, hidden_size=HID, intermediate_size=1024,
                      num_hidden_layers=LAYERS, num_attention_heads=HQ,
                      num_key_value_heads=HKV, head_dim=D, rope_theta=1e6,
                      max_position_embeddings=4096, initializer_range=0.08,
                      tie_word_embeddings=False)
    m = Qwen2ForCausalLM(cfg).to(torch.device("cuda:0"), torch.bfloat16).eval()
    return m


def _segments(q_lens, kv_visible, kv_total):
    """Segment dicts: block b's rows see ``kv_visible[b]`` (cached columns)
    and, causally, its own new rows (the last sum(q_lens) columns)."""
    from hsd_b200.plan import SEG_CAUSAL
    segs, q0 = [], 0
    for n, vis in zip(q_lens, kv_visible):
        kv = np.zeros(kv_total, dtype=bool)
        for a, b in vis:
            kv[a:b] = True
        segs.append({"q_start": q0, "q_len": n, "kind": SEG_CAUSAL, "kv": kv})
        q0 += n
    return segs


def _ours(m, ids, pos, plan, caches, base):
    """The package's path: rope + cache append, packed attention, fused argmax."""
    from hsd_b200.attention import flex_attention_forward
    from hsd_b200.lm_head import lm_head_argmax
    from hsd_b200.rope import rope_append
    q_len = ids.numel()
    kv_total = base + q_len
    h = m.model.embed_tokens(ids.long())[None]
    cos, sin = m.model.rotary_emb(h, pos[None])
    for l, layer in enumerate(m.model.layers):
        a = layer.self_attn
        x = layer.input_layernorm(h)
        q, k, v = a.q_proj(x)[0], a.k_proj(x)[0], a.v_proj(x)[0]
        kc, vc = caches[l]
        qv = rope_append(q.contiguous(), k.contiguous(), v.contiguous(), cos[0].contiguous(),
                         sin[0].contiguous(), kc, vc, base)
        o, _ = flex_attention_forward(a, qv, kc[None, :, :kv_total], vc[None, :, :kv_total],
                                      plan, a.scaling)
        h = h + a.o_proj(o.reshape(1, q_len, -1))
        h = h + layer.mlp(layer.post_attention_layernorm(h))
    return lm_head_argmax(m.model.norm(h)[0].contiguous(), m.lm_head.weight)


def _reference(m, ids, pos, allowed, ref_cache, base):
    """The reference's way on the same weights; returns (argmax ids, fp32 logits)."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    q_len = ids.numel()
    h = m.model.embed_tokens(ids.long())[None]
    cos, sin = m.model.rotary_emb(h, pos[None])
    neg = torch.where(torch.as_tensor(allowed, device=h.device), 0.0, float("-inf"))
    for l, layer in enumerate(m.model.layers):
        a = layer.self_attn
        x = layer.input_layernorm(h)
        q = a.q_proj(x).view(1, q_len, HQ, D).transpose(1, 2)
        k = a.k_proj(x).view(1, q_len, HKV, D).transpose(1, 2)
        v = a.v_proj(x).view(1, q_len, HKV, D).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        kc, vc = ref_cache[l]
        kc[:, base:base + q_len] = k[0]
        vc[:, base:base + q_len] = v[0]
        kk = kc[:, :base + q_len].float().repeat_interleave(HQ // HKV, 0)
        vv = vc[:, :base + q_len].float().repeat_interleave(HQ // HKV, 0)
        s = q[0].float() @ kk.transpose(1, 2) * a.scaling + neg[None]
        o = torch.nan_to_num(torch.softmax(s, -1)) @ vv
        o = o.to(torch.bfloat16).transpose(0, 1).reshape(1, q_len, -1)
        h = h + a.o_proj(o)
        h = h + layer.mlp(layer.post_attention_layernorm(h))
    logits = torch.nn.functional.linear(m.model.norm(h), m.lm_head.weight)[0]
    return logits.argmax(-1), logits.float()


def _compare(got, want, logits):
    diff = (got != want).nonzero().flatten().tolist()
    assert len(diff) <= max(1, int(0.03 * got.numel())), (len(diff), got.numel())
    for r in diff:
        best = logits[r, want[r]].item()
        assert logits[r, got[r]].item() >= best - 0.05 * (abs(best) + 1.0), r


def test_qwen2_prefill_and_verify_step(model):
    from hsd_b200.plan import PackedMask
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1, VOCAB, (n,), generator=g) for n in (70, 41, 96)]
    chunks = [torch.randint(1, VOCAB, (n,), generator=g) for n in (9, 17, 5)]
    cap = 512
    caches = [(torch.zeros(HKV, cap, D, dtype=torch.bfloat16, device=dev),
               torch.zeros(HKV, cap, D, dtype=torch.bfloat16, device=dev))
              for _ in range(LAYERS)]
    ref_caches = [(torch.zeros(HKV, cap, D, dtype=torch.bfloat16, device=dev),
                   torch.zeros(HKV, cap, D, dtype=torch.bfloat16, device=dev))
                  for _ in range(LAYERS)]
    with torch.no_grad():
        # step 1: packed prefill, block-diagonal causal
        ids1 = torch.cat(prompts).to(dev, torch.int32)
        pos1 = torch.cat([torch.arange(p.numel()) for p in prompts]).to(dev)
        q1 = ids1.numel()
        mask1 = PackedMask(q1, q1, _segments([p.numel() for p in prompts],
                                             [[]] * len(prompts), q1), device=dev)
        plan1 = mask1.plan()
        got1 = _ours(model, ids1, pos1, plan1, caches, 0)
        want1, logits1 = _reference(model, ids1, pos1, plan1.dense_allowed(), ref_caches, 0)
        torch.cuda.synchronize()
        _compare(got1, want1, logits1)
        # step 2: each block's new chunk sees its cached prompt and its own chunk causally
        starts = np.cumsum([0] + [p.numel() for p in prompts[:-1]]).tolist()
        ids2 = torch.cat(chunks).to(dev, torch.int32)
        pos2 = torch.cat([torch.arange(p.numel(), p.numel() + c.numel())
                          for p, c in zip(prompts, chunks)]).to(dev)
        q2, kv2 = ids2.numel(), q1 + ids2.numel()
        vis = [[(s, s + p.numel())] for s, p in zip(starts, prompts)]
        mask2 = PackedMask(q2, kv2, _segments([c.numel() for c in chunks], vis, kv2), device=dev)
        plan2 = mask2.plan()
        got2 = _ours(model, ids2, pos2, plan2, caches, q1)
        want2, logits2 = _reference(model, ids2, pos2, plan2.dense_allowed(), ref_caches, q1)
        torch.cuda.synchronize()
        _compare(got2, want2, logits2)
        # the caches hold the same rotated keys and values: bit-identical in
        # layer 0 (same inputs), within bf16 noise behind the first attention
        for l, ((kc, vc), (rk, rv)) in enumerate(zip(caches, ref_caches)):
            if l == 0:
                assert torch.equal(kc[:, :kv2], rk[:, :kv2])
                assert torch.equal(vc[:, :kv2], rv[:, :kv2])
            else:
                for a, b in ((kc, rk), (vc, rv)):
                    err = (a[:, :kv2].float() - b[:, :kv2].float()).abs().max().item()
                    assert err <= 0.05 * (b[:, :kv2].float().abs().max().item() + 1e-3)
