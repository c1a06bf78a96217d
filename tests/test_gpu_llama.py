"""Batched greedy decode of a Llama-architecture model on the paged cache
(metagross_b200/llama.py), small random-init shape.

* A decode step's logits equal, within fp16 rounding, the same step computed
  with dense fp32 attention over the cache's own dequantized K/V (gather):
  the cache integration (positions, rotary embedding, append before attend,
  GQA heads) is what differs.
* The CUDA-graph decode produces the same tokens as eager steps.
"""
import torch
import pytest

pytestmark = pytest.mark.gpu

SHAPE = dict(vocab=512, hidden=512, layers=2, heads=8, kv_heads=2, ffn=512)  # head_dim 64


def _decoder(kv="int8", keep=True):
    from metagross_b200.llama import LlamaDecoder, LlamaShape

    return LlamaDecoder(LlamaShape(**SHAPE), batch=3, max_len=64, kv_dtype=kv, seed=5, keep_logits=keep)


def _prompt():
    g = torch.Generator().manual_seed(9)
    return torch.randint(0, SHAPE["vocab"], (3, 21), generator=g)


def _reference_logits(dec, ids, pos):
    """The decode step of ids at positions pos, attention over cache.gather in fp32."""
    s = dec.s
    x = dec.w["embed"][ids]
    rep = s.heads // s.kv_heads
    for i in range(s.layers):
        q, k, v = dec._qkv(i, dec._rms(x, dec.w[f"{i}.n1"]))
        q = dec._rope(q, pos)
        kc, vc, cu = dec.cache.gather(i, dtype=torch.float32)
        o = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        for b in range(dec.batch):
            K = kc[int(cu[b]):int(cu[b + 1])].repeat_interleave(rep, dim=1)  # [T, Hq, D]
            V = vc[int(cu[b]):int(cu[b + 1])].repeat_interleave(rep, dim=1)
            sc = torch.einsum("hd,thd->ht", q[b].float(), K) / s.head_dim ** 0.5
            o[b] = torch.einsum("ht,thd->hd", torch.softmax(sc, dim=-1), V)
        x = x + o.to(x.dtype).flatten(1) @ dec.w[f"{i}.wo"]
        x = dec._mlp(i, x)
    return dec._logits(x).float()


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_decode_step_matches_dense_attention_over_the_cache(kv):
    dec = _decoder(kv)
    dec.prefill(_prompt().cuda())
    for _ in range(4):
        ids, pos = dec.ids.clone(), dec.pos.clone()
        dec._step()
        dec.cache.check()
        ref = _reference_logits(dec, ids, pos)
        got = dec.logits.float()
        err = (got - ref).abs().max().item()
        assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


def test_graph_decode_equals_eager():
    a, b = _decoder(keep=False), _decoder(keep=False)
    p = _prompt().cuda()
    a.prefill(p)
    b.prefill(p)
    b.capture()
    ta = a.decode(20)
    tb = b.decode(20)
    a.cache.check()
    b.cache.check()
    assert torch.equal(ta, tb)
    assert int(a.pos[0]) == 21 + 19 and torch.equal(a.pos, b.pos)


def test_fused_dense_ops_match_torch():
    from metagross_b200 import _C

    g = torch.Generator(device="cuda").manual_seed(3)
    for cols in (384, 2048, 5000, 100):  # register paths (one / four 2048-column groups) and the general one
        x = torch.randn(7, cols, generator=g, device="cuda").half()
        w = (1 + 0.1 * torch.randn(cols, generator=g, device="cuda")).half()
        x32 = x.float()
        ref = (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + 1e-5)).half() * w
        assert (_C.rmsnorm(x, w, 1e-5).float() - ref.float()).abs().max().item() <= 4e-3, cols
    for F in (96, 100):  # 8-wide and scalar paths
        gu = torch.randn(5, 2 * F, generator=g, device="cuda").half()
        ref = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        assert (_C.silu_mul(gu).float() - ref.float()).abs().max().item() <= 4e-3, F
    B, Hq, Hkv, D = 4, 8, 2, 64
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g, device="cuda").half()
    pos = torch.tensor([0, 3, 17, 40], device="cuda")
    ang = torch.outer(torch.arange(64, device="cuda").float(), 1.0 / 10000 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q, k = torch.empty(B, Hq, D, device="cuda").half(), torch.empty(B, Hkv, D, device="cuda").half()
    v = torch.empty_like(k)
    _C.rope_qkv(qkv, pos, cos, sin, q, k, v)
    qq, kk, vv = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)

    def rot(t, n):
        t = t.view(B, n, D).float()
        c, s_ = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
        return torch.cat([t[..., :32] * c - t[..., 32:] * s_, t[..., 32:] * c + t[..., :32] * s_], -1).half()

    assert (q.float() - rot(qq, Hq).float()).abs().max().item() <= 2e-3
    assert (k.float() - rot(kk, Hkv).float()).abs().max().item() <= 2e-3
    assert torch.equal(v, vv.reshape(B, Hkv, D))


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_fused_rotary_append_equals_rotary_then_append(kv):
    """mg_kv_append_rope against mg_rope_qkv_f16 + mg_kv_append on twin caches:
    pools, scales, staging and block tables bit for bit, and the same rotated
    q, over a prefill-sized step (page commits) and decode steps."""
    from metagross_b200 import _C
    from metagross_b200.batched import BatchedPagedKVCache

    B, Hq, Hkv, D, P = 3, 8, 2, 64, 16
    g = torch.Generator(device="cuda").manual_seed(21)
    ang = torch.outer(torch.arange(128, device="cuda").float(),
                      1.0 / 10000 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    mk = lambda: BatchedPagedKVCache(1, B, Hkv, D, page_size=P, num_pages=32, max_blocks=8, kv_dtype=kv)  # noqa: E731
    fused, plain = mk(), mk()
    for T in (37, 1, 1, 5, 1):
        n = torch.randint(0, T + 1, (B,), generator=torch.Generator().manual_seed(T), dtype=torch.int32)
        qkv = torch.randn(B, T, (Hq + 2 * Hkv) * D, generator=g, device="cuda").half()
        lens = fused.seq_lens.long()
        pos = (lens[:, None] + torch.arange(T, device="cuda")[None]).reshape(-1)
        q_plain = torch.empty(B * T, Hq, D, device="cuda").half()
        k_plain = torch.empty(B * T, Hkv, D, device="cuda").half()
        v_plain = torch.empty_like(k_plain)
        _C.rope_qkv(qkv.reshape(B * T, -1), pos, cos, sin, q_plain, k_plain, v_plain)
        for c in (fused, plain):
            c.begin_step(n)
        q_fused = torch.zeros(B, T, Hq, D, device="cuda").half()
        fused.append_rope(0, qkv, Hq, cos, sin, q_fused)
        plain.append(0, k_plain.view(B, T, Hkv, D), v_plain.view(B, T, Hkv, D))
        torch.cuda.synchronize()
        fused.check()
        plain.check()
        for name in ("k_pool", "v_pool", "k_scales", "v_scales", "staging_k", "staging_v", "block_tables",
                     "seq_lens"):
            assert torch.equal(getattr(fused, name), getattr(plain, name)), (T, name)
        qp = q_plain.view(B, T, Hq, D)
        for b in range(B):
            assert torch.equal(q_fused[b, :int(n[b])], qp[b, :int(n[b])]), (T, b)


def test_fused_rotary_decoder_equals_unfused():
    from metagross_b200.llama import LlamaDecoder, LlamaShape

    p = _prompt().cuda()
    toks = []
    for fused in (True, False):
        d = LlamaDecoder(LlamaShape(**SHAPE), batch=3, max_len=64, kv_dtype="int8", seed=5, fused_rope=fused)
        d.prefill(p)
        d.capture()
        toks.append(d.decode(16))
        d.cache.check()
    assert torch.equal(toks[0], toks[1])


def test_fused_rotary_append_flags_a_position_beyond_the_table():
    from metagross_b200.batched import BatchedPagedKVCache

    B, Hq, Hkv, D = 2, 4, 2, 64
    c = BatchedPagedKVCache(1, B, Hkv, D, page_size=16, num_pages=8, max_blocks=4)
    cos = torch.ones(4, D // 2, device="cuda")
    sin = torch.zeros(4, D // 2, device="cuda")
    qkv = torch.randn(B, 6, (Hq + 2 * Hkv) * D, device="cuda").half()
    c.begin_step(6)  # positions 0..5, the table has 4 rows
    c.append_rope(0, qkv, Hq, cos, sin, torch.empty(B, 6, Hq, D, device="cuda").half())
    torch.cuda.synchronize()
    assert int(c.status.item()) & 0x80
