"""A whole batch-1 decode step under one CUDA graph (decode_step.DecodeStack;
the reference's serving/cudagraph.py): graph replays equal the eager static
step bit for bit, token after token, and the logits track a float32
recomputation from the decoded weights."""
from __future__ import annotations

import pytest
import torch

from drinkme_b200 import decode_step

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SMALL = dict(layers=2, hidden=1024, inter=2048, heads=8, kv_heads=2, head_dim=128, vocab=1000)


def test_graph_replay_equals_eager_and_tracks_float32():
    eager = decode_step.DecodeStack(SMALL, DEV, max_len=32, seed=1)
    graphed = decode_step.DecodeStack(SMALL, DEV, max_len=32, seed=1)
    for st in (eager, graphed):
        st.reset(token=7)
    graphed.capture()
    fed = []
    for _ in range(6):
        fed.append(int(eager.token))
        eager.step()
        graphed.replay()
        torch.cuda.synchronize()
        assert torch.equal(eager.logits, graphed.logits)
        assert torch.equal(eager.token, graphed.token) and torch.equal(eager.pos, graphed.pos)
    ref = eager.reference_logits(fed)
    got = graphed.logits.float()
    assert (got - ref).norm() / ref.norm() < 3e-2  # bf16 activations between the ops vs float32
    top2 = torch.topk(ref[0], 2).values
    if float(top2[0] - top2[1]) > 0.05 * float(ref.abs().max()):
        assert int(got.argmax()) == int(ref.argmax())


@pytest.mark.parametrize("nh,nkv", [(8, 2), (64, 8)])
def test_attention_block_equals_two_launches(nh, nkv):
    """dm_step_attention_block (one launch) gives the same bits as
    dm_step_qk_rope_cache followed by dm_step_attention: the attention
    output and both cache rows, at positions on and beside chunk edges."""
    import ctypes as ct

    from drinkme_b200 import _lib, radix_ops

    hd, max_len = 128, 400
    g = torch.Generator(device=DEV).manual_seed(5)

    def rnd(*size, scale=1.0):
        return (torch.randn(size, generator=g, device=DEV) * scale).to(torch.bfloat16)

    qn, kn = (1 + rnd(hd, scale=0.1).float()).bfloat16(), (1 + rnd(hd, scale=0.1).float()).bfloat16()
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float32) / hd))
    ang = torch.arange(max_len, device=DEV, dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    L = _lib.lib()
    work2 = torch.zeros(int(L.dm_step_attention_workspace_bytes(nh, hd, max_len)) // 4 + 1, device=DEV)
    work1 = torch.zeros(int(L.dm_step_attention_block_workspace_bytes(nh, nkv, hd, max_len)) // 4 + 1, device=DEV)
    kc1, vc1 = rnd(max_len, nkv, hd), rnd(max_len, nkv, hd)
    kc2, vc2 = kc1.clone(), vc1.clone()
    st = radix_ops._stream(DEV)
    P = ct.c_void_p

    def ptr(t):
        return P(t.data_ptr())

    for p in (0, 1, 31, 32, 33, 127, 128, 129, 255, 256, 399):
        qkv = rnd(1, (nh + 2 * nkv) * hd)
        pos = torch.tensor([p], dtype=torch.int64, device=DEV)
        q = torch.empty(nh, hd, dtype=torch.bfloat16, device=DEV)
        out1 = torch.empty(1, nh * hd, dtype=torch.bfloat16, device=DEV)
        out2 = torch.empty_like(out1)
        _lib.call("dm_step_qk_rope_cache", ptr(qkv), ptr(qn), ptr(kn), ptr(cos), ptr(sin), ptr(pos), ptr(q),
                  ptr(kc2), ptr(vc2), nh, nkv, hd, ct.c_float(1e-6), st)
        _lib.call("dm_step_attention", ptr(q), ptr(kc2), ptr(vc2), ptr(pos), max_len, ptr(out2), ptr(work2),
                  nh, nkv, hd, st)
        _lib.call("dm_step_attention_block", ptr(qkv), ptr(qn), ptr(kn), ptr(cos), ptr(sin), ptr(pos), ptr(kc1),
                  ptr(vc1), max_len, ptr(out1), ptr(work1), nh, nkv, hd, ct.c_float(1e-6), st)
        torch.cuda.synchronize()
        assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2), p
        assert torch.equal(out1, out2), p
        assert bool(torch.isfinite(out1.float()).all())
