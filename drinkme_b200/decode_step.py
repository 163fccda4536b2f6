"""A whole batch-1 decode step of a Qwen3-shaped decoder stack, its packed
Linears served by this package's kernels, captured in one CUDA graph — the
analogue of the reference's graphed decode step (src/drinkme/serving/
cudagraph.py: one torch.cuda.CUDAGraph per step, every input on the device,
the live length a device counter, the KV rows written inside the graph).

Per layer: RMSNorm; the fused q|k|v GEMV (one sip tensor handle, radix_ops.
gemv_into); per-head RMSNorm of q and k (Qwen3's q_norm / k_norm); rotary
embedding at the device position; the new K/V row written into a static
cache; grouped-query attention over the cache's live rows (their count read
from the device position, so one graph serves every length up to the
allocation); the
o GEMV and the residual add; RMSNorm; the fused gate|up GEMV; SiLU(gate) *
up; the down GEMV and the residual add. Then the final RMSNorm, the raw
bf16 lm_head (radix_ops.gemv_raw's kernel), a greedy argmax written back
into the token buffer, and the position advanced — so replaying the graph
decodes token after token with no host work.

The Linears are the hot path (the sip GEMV, the raw lm_head GEMV); the
operations between them are this package's small fused kernels (csrc/
step_ops.cu: residual add + RMSNorm; the attention block — q/k RMSNorm,
rotary, KV-cache write, split-K decode attention and its combine — in one
launch; SiLU * up) — eight launches per layer; the
reference runs transformers' own modules there. The embedding lookup, the
greedy argmax and the position counter are torch operations. Weights are synthetic (random N(0, 0.02),
packed sip by this package's encoder); `reference_logits` recomputes one
step in float32 from the decoded weights for the parity check.
"""
from __future__ import annotations

import ctypes as ct
import math

import torch

from . import _lib, codec, radix_ops, swap

QWEN3 = {
    "qwen3-8b": dict(layers=36, hidden=4096, inter=12288, heads=32, kv_heads=8, head_dim=128, vocab=151936),
    "qwen3-32b": dict(layers=64, hidden=5120, inter=25600, heads=64, kv_heads=8, head_dim=128, vocab=151936),
}
EPS = 1e-6
ROPE_THETA = 1e6


class DecodeStack:
    """Static buffers and packed weights for one batch-1 decode step; see the
    module docstring. `variants` distinct packed tensors per shape are
    cloned across the layers (every layer its own HBM copy)."""

    def __init__(self, shape: dict, device="cuda", max_len: int = 1024, seed: int = 0, variants: int = 2,
                 layers: int | None = None):
        dev = torch.device(device)
        self.dev, self.s = dev, dict(shape)
        if layers is not None:
            self.s["layers"] = layers
        s = self.s
        H, I, nh, nkv, hd = s["hidden"], s["inter"], s["heads"], s["kv_heads"], s["head_dim"]
        self.max_len = max_len
        g = torch.Generator(device=dev).manual_seed(seed)

        def rnd(*size, scale=0.02):
            return (torch.randn(size, generator=g, device=dev) * scale).to(torch.bfloat16)

        def pack(w):
            return codec.pack_array_radix_device(w.view(torch.int16), "sip")

        protos = []
        for _ in range(max(1, variants)):
            q, k, v = rnd(nh * hd, H), rnd(nkv * hd, H), rnd(nkv * hd, H)
            gate, up = rnd(I, H), rnd(I, H)
            protos.append({
                "qkv": swap.to_device_radix_fused([pack(q), pack(k), pack(v)], dev),
                "o": swap.to_device_radix(pack(rnd(H, nh * hd)), dev),
                "gate_up": swap.to_device_radix_fused([pack(gate), pack(up)], dev),
                "down": swap.to_device_radix(pack(rnd(H, I)), dev),
            })
            del q, k, v, gate, up

        def clone(rt):
            return dict(rt, rx_handle=rt["rx_handle"].clone())

        self.layers = []
        for li in range(s["layers"]):
            p = protos[li % len(protos)]
            lay = {k: (p[k] if li < len(protos) else clone(p[k])) for k in p}
            lay["ln1"] = (1.0 + rnd(H, scale=0.1).float()).to(torch.bfloat16)
            lay["ln2"] = (1.0 + rnd(H, scale=0.1).float()).to(torch.bfloat16)
            lay["qn"] = (1.0 + rnd(hd, scale=0.1).float()).to(torch.bfloat16)
            lay["kn"] = (1.0 + rnd(hd, scale=0.1).float()).to(torch.bfloat16)
            self.layers.append(lay)
        self.embed = rnd(s["vocab"], H, scale=1.0)
        self.norm = (1.0 + rnd(H, scale=0.1).float()).to(torch.bfloat16)
        self.head = rnd(s["vocab"], H)
        L = s["layers"]
        self.kcache = torch.zeros(L, max_len, nkv, hd, dtype=torch.bfloat16, device=dev)
        self.vcache = torch.zeros(L, max_len, nkv, hd, dtype=torch.bfloat16, device=dev)
        inv = 1.0 / (ROPE_THETA ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
        ang = torch.arange(max_len, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos(), ang.sin()  # [max_len, hd / 2]
        # the step's device state: the token to feed, the position to write
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.logits = torch.empty(1, s["vocab"], dtype=torch.bfloat16, device=dev)
        # static activations
        self.h = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        self.x = torch.empty(1, H, dtype=torch.bfloat16, device=dev)  # the normed input of the next Linear
        self.q = torch.empty(nh, hd, dtype=torch.bfloat16, device=dev)
        self.work = torch.zeros(int(_lib.lib().dm_step_attention_block_workspace_bytes(nh, nkv, hd, max_len)) // 4 + 1,
                                dtype=torch.float32, device=dev)
        self.qkv = torch.empty(1, (nh + 2 * nkv) * hd, dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty(1, nh * hd, dtype=torch.bfloat16, device=dev)
        self.o = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        self.gu = torch.empty(1, 2 * I, dtype=torch.bfloat16, device=dev)
        self.act = torch.empty(1, I, dtype=torch.bfloat16, device=dev)
        self.dn = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        self.graph = None

    # -- one step, eager; every tensor it touches is static -----------------
    def step(self) -> None:
        s = self.s
        nh, nkv, hd, H, I = s["heads"], s["kv_heads"], s["head_dim"], s["hidden"], s["inter"]
        st = radix_ops._stream(self.dev)
        P = ct.c_void_p

        def ptr(t):
            return P(t.data_ptr())

        self.h.copy_(self.embed.index_select(0, self.token))
        delta = None
        for li, lay in enumerate(self.layers):
            _lib.call("dm_step_add_rmsnorm", ptr(self.h), ptr(delta) if delta is not None else P(0), ptr(lay["ln1"]),
                      ptr(self.x), H, ct.c_float(EPS), st)
            radix_ops.gemv_into(lay["qkv"], self.x, None, self.qkv)
            _lib.call("dm_step_attention_block", ptr(self.qkv), ptr(lay["qn"]), ptr(lay["kn"]), ptr(self.cos),
                      ptr(self.sin), ptr(self.pos), ptr(self.kcache[li]), ptr(self.vcache[li]), self.max_len,
                      ptr(self.attn), ptr(self.work), nh, nkv, hd, ct.c_float(EPS), st)
            radix_ops.gemv_into(lay["o"], self.attn, None, self.o)
            _lib.call("dm_step_add_rmsnorm", ptr(self.h), ptr(self.o), ptr(lay["ln2"]), ptr(self.x), H,
                      ct.c_float(EPS), st)
            radix_ops.gemv_into(lay["gate_up"], self.x, None, self.gu)
            _lib.call("dm_step_silu_mul", ptr(self.gu), ptr(self.act), I, st)
            radix_ops.gemv_into(lay["down"], self.act, None, self.dn)
            delta = self.dn
        _lib.call("dm_step_add_rmsnorm", ptr(self.h), ptr(delta) if delta is not None else P(0), ptr(self.norm),
                  ptr(self.x), H, ct.c_float(EPS), st)
        _lib.call("dm_gemv_raw", ptr(self.head), s["vocab"], H, ptr(self.x), _lib.DM_BF16, 1, P(0), ptr(self.logits),
                  _lib.DM_BF16, st)
        torch.argmax(self.logits, -1, out=self.token)
        self.pos.add_(1)

    # -- the graph ----------------------------------------------------------
    def capture(self) -> None:
        """Capture one step (after a warm-up step on a side stream, whose
        cache row and position are then rewound)."""
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        tok, pos = self.token.clone(), self.pos.clone()
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        self.token.copy_(tok)
        self.pos.copy_(pos)
        torch.cuda.synchronize(self.dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.step()
        torch.cuda.synchronize(self.dev)

    def replay(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def reset(self, token: int = 0) -> None:
        self.token.fill_(int(token))
        self.pos.zero_()
        self.kcache.zero_()
        self.vcache.zero_()

    # -- parity ---------------------------------------------------------------
    def reference_logits(self, tokens: list[int]) -> torch.Tensor:
        """float32 logits of the last position after feeding `tokens` one by
        one, recomputed from the decoded weights with dense matmuls."""
        s = self.s
        nh, nkv, hd = s["heads"], s["kv_heads"], s["head_dim"]
        grp = nh // nkv
        W = [{k: radix_ops.decode_weight(lay[k]).float() for k in ("qkv", "o", "gate_up", "down")}
             for lay in self.layers]
        Ks = [[] for _ in self.layers]
        Vs = [[] for _ in self.layers]

        def rms(x, w):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS) * w.float()

        def rope(x, p):
            c, sn = self.cos[p], self.sin[p]
            h = x.shape[-1] // 2
            return torch.cat([x[..., :h] * c - x[..., h:] * sn, x[..., h:] * c + x[..., :h] * sn], -1)

        logits = None
        for p, t in enumerate(tokens):
            h = self.embed[t].float()[None]
            for li, lay in enumerate(self.layers):
                qkv = rms(h, lay["ln1"]) @ W[li]["qkv"].T
                q = rope(rms(qkv[0, : nh * hd].view(nh, hd), lay["qn"]), p)
                k = rope(rms(qkv[0, nh * hd: (nh + nkv) * hd].view(nkv, hd), lay["kn"]), p)
                v = qkv[0, (nh + nkv) * hd:].view(nkv, hd)
                Ks[li].append(k)
                Vs[li].append(v)
                K = torch.stack(Ks[li], 1)  # [nkv, p + 1, hd]
                V = torch.stack(Vs[li], 1)
                sc = torch.matmul(q.view(nkv, grp, hd), K.transpose(1, 2)) / math.sqrt(hd)
                att = torch.matmul(torch.softmax(sc, -1), V).reshape(1, nh * hd)
                h = h + att @ W[li]["o"].T
                gu = rms(h, lay["ln2"]) @ W[li]["gate_up"].T
                h = h + (torch.nn.functional.silu(gu[:, : s["inter"]]) * gu[:, s["inter"]:]) @ W[li]["down"].T
            logits = rms(h, self.norm) @ self.head.float().T
        return logits


def main(argv=None) -> int:
    """`python -m drinkme_b200.decode_step`: device time per token of the
    graphed Qwen3-8B-shaped step (synthetic weights), at positions from
    `--position` on."""
    import argparse
    import json

    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=tuple(QWEN3), default="qwen3-8b")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--position", type=int, default=0)
    ap.add_argument("--max-len", type=int, default=1024)
    a = ap.parse_args(argv)
    st = DecodeStack(QWEN3[a.shape], "cuda:0", max_len=a.max_len, seed=11)
    st.reset(token=1)
    st.capture()
    st.pos.fill_(a.position)
    for _ in range(a.warmup):
        st.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(a.steps):
        st.replay()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / a.steps
    print(json.dumps({"shape": a.shape, "position": a.position, "steps": a.steps, "ms_per_step": round(ms, 4),
                      "tokens_per_s": round(1e3 / ms, 2)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
