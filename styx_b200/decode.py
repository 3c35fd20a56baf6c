"""One decode step of the MoE model on one device: MoeModel::forward_token
(crates/model/src/moe.rs:1780-2140) and generate_moe's greedy loop
(crates/model/examples/generate_moe.rs:29-66), composed from the library's
kernels through the C ABI.

Per token: the embedding row (styx_get_rows), then per layer the attention
half (styx_attn_block: RMSNorm, q/k/v, per-head norms, RoPE, the KV cache
row, attention, o, residual) and the MoE block (styx_moe_block), then the
output norm, the LM head GEMV and the greedy pick on the device
(styx_argmax_f32).  The KV caches hold n_ctx positions at most: allocated
once (kv_page 0), or grown page by page as the reference does
(moe.rs:501-503, 1802-1822: pages of KV_PAGE_TOKENS = 512 rows, every
layer's caches reallocated one page larger and the filled rows copied over
-- here a device-to-device copy on the stream instead of a host round trip);
the attention reads the same rows either way, so the results are the same
bits.

Expert parallelism (`allreduce` or `ep_comm` given): every rank runs the
whole step on the same token with the same dense weights, but holds only
its own experts (its layers' hot buffers, remap -> local slot); each MoE
block writes its slot contributions (styx_moe_block_ep), `allreduce` sums
them over the ranks in place on the stream and styx_moe_combine adds the
slot-ordered sum into x, or `ep_comm` (ops.EpComm) does the exchange over
NVLink peer memory -- by default inside the block's own kernel
(styx_ep_moe_block), else as one kernel after it -- either way bit-identical
to one device holding every expert.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch

from . import ops


@dataclass
class DecodeParams:
    """HParams (moe.rs:550-587) of a Qwen3-MoE model."""
    n_layers: int
    n_embd: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    n_vocab: int
    rms_eps: float = 1e-6
    rope_base: float = 1_000_000.0
    norm_topk: bool = True
    qk_norm: bool = True


@dataclass
class DecodeLayer:
    attn: ops.AttnWeights
    moe: ops.LayerWeights


class DecodeModel:
    def __init__(self, hp: DecodeParams, embd: ops.DenseWeight, layers: list, output_norm: torch.Tensor,
                 head: ops.DenseWeight, n_ctx: int, device: int = 0, allreduce=None, kv_page: int = 0,
                 ep_comm=None, ep_fused: bool = True):
        self.hp, self.embd, self.layers, self.output_norm, self.head = hp, embd, layers, output_norm, head
        self.n_ctx = n_ctx            # n_ctx_max: positions the caches may grow to
        self.kv_page = kv_page        # 0: allocated once for n_ctx rows; else rows per page
        dev = f"cuda:{device}"
        self.attn = ops.AttnBlock(hp.n_embd, hp.n_heads, hp.n_kv_heads, hp.head_dim, hp.qk_norm, hp.rms_eps,
                                  hp.rope_base, device)
        self.moe = ops.MoeBlock(ops.Dims(hp.n_embd, hp.n_ff, hp.n_expert, hp.n_expert_used, hp.norm_topk,
                                         hp.rms_eps), device)
        kv_dim = hp.n_kv_heads * hp.head_dim
        self.cap = min(n_ctx, kv_page) if kv_page > 0 else n_ctx   # rows the caches hold now
        self.kcache = torch.zeros(hp.n_layers, self.cap, kv_dim, dtype=torch.float32, device=dev)
        self.vcache = torch.zeros_like(self.kcache)
        self.x = torch.empty(hp.n_embd, dtype=torch.float32, device=dev)
        self.xn = torch.empty_like(self.x)
        self.logits = torch.empty(hp.n_vocab, dtype=torch.float32, device=dev)
        self.ids = torch.zeros(hp.n_layers * ops.IDS_PER_LAYER, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.next = torch.zeros(1, dtype=torch.int32, device=dev)
        self.n_past = 0
        # expert parallelism: a callable summing a tensor over the ranks in
        # place, on the current stream (e.g. torch.distributed.all_reduce)
        self.allreduce = allreduce
        # or: an ops.EpComm (the exchange over NVLink peer memory): with
        # ep_fused the block and the exchange in one call (styx_ep_moe_block:
        # one kernel where the single-kernel form fits), else the block's
        # partial then styx_ep_combine
        self.ep_comm = ep_comm
        self.ep_fused = ep_fused
        self.partial = torch.zeros(hp.n_expert_used * hp.n_embd, dtype=torch.float32, device=dev)

    def _grow(self) -> None:
        """One page more for every layer's K and V caches (moe.rs:1802-1822):
        new buffers, the filled rows copied, the old ones released (on the
        current stream, so the copy is ordered after every earlier step)."""
        cap = min(self.n_ctx, self.cap + self.kv_page)
        for name in ("kcache", "vcache"):
            old = getattr(self, name)
            new = torch.zeros(old.shape[0], cap, old.shape[2], dtype=old.dtype, device=old.device)
            new[:, :self.cap].copy_(old)
            setattr(self, name, new)
        self.cap = cap

    def reset(self) -> None:
        self.n_past = 0

    def forward_token(self, token: int, stream=None) -> torch.Tensor:
        """Runs one token at position n_past; returns the device logits
        (and leaves the greedy pick in self.next)."""
        if self.n_past >= self.n_ctx:
            raise ValueError(f"KV caches full ({self.n_ctx})")
        with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
            if self.n_past >= self.cap:
                self._grow()
            self.tok.fill_(token)
            self.pos.fill_(self.n_past)
        self.step(stream)
        self.n_past += 1
        return self.logits

    def step(self, stream=None) -> None:
        """The kernels of one token: the token id in self.tok and its position
        in self.pos (device) and self.n_past (host, the attention's row
        count) are the caller's; n_past is not advanced.  Everything here is
        stream-ordered launches, so a graph can record it."""
        hp, pos = self.hp, self.n_past
        ops.get_rows(self.embd.qtype, self.embd.data, hp.n_vocab, hp.n_embd, self.tok, out=self.x, stream=stream)
        for li, ly in enumerate(self.layers):
            self.attn.forward(self.x, ly.attn, pos, self.pos, self.kcache[li], self.vcache[li], self.cap,
                              stream=stream)
            if self.ep_comm is not None and self.ep_fused:
                self.ep_comm.moe_block(self.moe, self.x, ly.moe, li, self.ids, stream=stream)
            elif self.ep_comm is not None:
                self.moe.forward_ep(self.x, ly.moe, li, self.ids, self.partial, stream=stream)
                self.ep_comm.combine(self.partial, self.x, stream=stream)
            elif self.allreduce is None:
                self.moe.forward(self.x, ly.moe, li, self.ids, stream=stream)
            else:
                self.moe.forward_ep(self.x, ly.moe, li, self.ids, self.partial, stream=stream)
                with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
                    self.allreduce(self.partial)
                self.moe.combine(self.partial, self.x, stream=stream)
        ops.rms_norm_into(self.x, self.output_norm, hp.rms_eps, self.xn, stream=stream)
        ops.mul_mat_vec(self.head.qtype, self.head.data, hp.n_vocab, hp.n_embd, self.xn, y=self.logits,
                        stream=stream)
        ops.argmax_f32(self.logits, out=self.next, stream=stream)

    def generate(self, prompt: list, n_predict: int, stream=None) -> list:
        """generate_moe's loop (examples/generate_moe.rs:46-66): the prompt
        token by token, then n_predict greedy tokens, each the argmax of the
        previous step's logits (n_predict - 1 further steps)."""
        assert prompt and n_predict > 0, "empty prompt or nothing to predict"
        for t in prompt:
            self.forward_token(t, stream)
        out = [int(self.next.item())]
        for _ in range(1, n_predict):
            self.forward_token(out[-1], stream)
            out.append(int(self.next.item()))
        return out
