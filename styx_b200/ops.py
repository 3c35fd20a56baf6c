"""Torch-facing wrappers of the styx MoE-block operators.

Each function mirrors one dispatch that MoeModel::forward_token records for
the MoE block (crates/model/src/moe.rs:1974-2062) and calls the sm_100a
kernels of libstyx_moe.so through its C ABI.  Device tensors are passed by
pointer; work is queued on torch's current CUDA stream.  There is no CPU
path: without the library or a GPU these functions raise.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional

import torch

from . import _lib
from ._lib import (BLOCK, IDS_PER_LAYER, Q4_K, Q5_K, Q6_K, Q8_0, SKIP, ExpertTensor,  # noqa: F401
                   MoeDims, MoeLayer, StyxError, check, lib, row_bytes)

_ctxs: dict[int, "Context"] = {}


class Context:
    """styx_ctx for one CUDA device (Gpu::new, crates/vk-backend/src/lib.rs:356)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = C.c_void_p()
        check(lib().styx_init(device, C.byref(h)))
        self.handle = h
        n = C.c_int()
        name = C.create_string_buffer(256)
        check(lib().styx_device_info(h, C.byref(n), name, 256))
        self.sm_count = n.value
        self.name = name.value.decode()

    def vram_bytes(self) -> int:
        v = C.c_uint64()
        check(lib().styx_vram_bytes(self.handle, C.byref(v)))
        return v.value

    def check_device_error(self, stream=None) -> None:
        check(lib().styx_check_device_error(self.handle, _stream(stream)))

    def set_option(self, option: int, value: int) -> None:
        check(lib().styx_set_option(self.handle, option, value))

    def get_option(self, option: int) -> int:
        v = C.c_int64()
        check(lib().styx_get_option(self.handle, option, C.byref(v)))
        return v.value

    def set_moe_kernels(self, mode: int) -> None:
        """0 auto, 1 the single cooperative kernel, 2 three kernels, 3 the cluster form."""
        self.set_option(_lib.OPT_MOE_KERNELS, mode)

    def last_moe_path(self) -> int:
        """1 = single kernel, 2 = three kernels, 3 = host-read form, 4 / 5 = single
        kernel over several layers, 6 = cluster form (the last styx_moe_block[s])."""
        return self.get_option(_lib.OPT_MOE_LAST_PATH)


def ctx(device: Optional[int] = None) -> Context:
    if device is None:
        device = torch.cuda.current_device()
    if device not in _ctxs:
        _ctxs[device] = Context(device)
    return _ctxs[device]


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def _dev(t: torch.Tensor) -> int:
    assert t.is_cuda, "styx ops take CUDA tensors"
    return t.device.index


class HostBuffer:
    """Pinned, device-mapped host memory (STYX_MEM_HOST, the GTT tier of
    create_buffer_host_shared, lib.rs:802).  `.tensor` is a CPU uint8 view
    whose data_ptr the kernels can read."""

    def __init__(self, nbytes: int, device: Optional[int] = None):
        self.ctx = ctx(device)
        p = C.c_void_p()
        check(lib().styx_alloc(self.ctx.handle, nbytes, _lib.MEM_HOST, C.byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes
        arr = (C.c_uint8 * nbytes).from_address(self.ptr)
        self.tensor = torch.frombuffer(arr, dtype=torch.uint8)

    def free(self) -> None:
        if self.ptr:
            self.tensor = None
            check(lib().styx_free(self.ctx.handle, C.c_void_p(self.ptr)))
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ------------------------------------------------------------------ ops
def rms_norm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    nrows = 1 if x.dim() == 1 else x.shape[0]
    out = torch.empty_like(x)
    check(lib().styx_rms_norm(ctx(_dev(x)).handle, _stream(), _ptr(x), _ptr(w), eps, x.shape[-1], nrows,
                              _ptr(out)))
    return out


def rms_norm_into(x: torch.Tensor, w: Optional[torch.Tensor], eps: float, out: torch.Tensor,
                  stream=None) -> torch.Tensor:
    """rms_norm_f32 over the last dimension into `out` on `stream`."""
    nrows = 1 if x.dim() == 1 else x.shape[0]
    check(lib().styx_rms_norm(ctx(_dev(x)).handle, _stream(stream), _ptr(x), _ptr(w), eps, x.shape[-1], nrows,
                              _ptr(out)))
    return out


def matvec_f32(a: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    d = torch.empty(a.shape[0], dtype=torch.float32, device=a.device)
    check(lib().styx_matvec_f32(ctx(_dev(a)).handle, _stream(), _ptr(a), a.shape[0], a.shape[1], a.stride(0),
                                _ptr(x), _ptr(d)))
    return d


def topk_softmax(logits: torch.Tensor, k: int, renorm: bool = True, remap: Optional[torch.Tensor] = None,
                 pmap: Optional[torch.Tensor] = None):
    """-> (weights f32[k], ids64 i32[64]) (shaders/topk_softmax_f32.comp)."""
    w = torch.empty(k, dtype=torch.float32, device=logits.device)
    ids = torch.full((IDS_PER_LAYER,), -1, dtype=torch.int32, device=logits.device)
    check(lib().styx_topk_softmax(ctx(_dev(logits)).handle, _stream(), _ptr(logits), logits.numel(), k,
                                  int(renorm), _ptr(remap), _ptr(pmap), _ptr(w), _ptr(ids)))
    return w, ids


def mul_mat_vec_id(qtype: int, a: torch.Tensor, expert_bytes: int, nrows: int, ncols: int, ids: torch.Tensor,
                   x: torch.Tensor, ne11: int, y: Optional[torch.Tensor] = None,
                   n_expert: Optional[int] = None) -> torch.Tensor:
    """y[s*nrows + r] = deq(A[ids[s]])[r] . x[s % ne11] (MatVecIdPush semantics)."""
    n_ids = ids.numel()
    if n_expert is None:
        n_expert = a.numel() // expert_bytes
    if y is None:
        y = torch.zeros(n_ids * nrows, dtype=torch.float32, device=a.device)
    check(lib().styx_mul_mat_vec_id(ctx(_dev(a)).handle, _stream(), qtype, _ptr(a), expert_bytes, n_expert, nrows,
                                    ncols, _ptr(ids), n_ids, _ptr(x), ncols, ne11, _ptr(y), nrows))
    return y


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(g)
    check(lib().styx_swiglu(ctx(_dev(g)).handle, _stream(), _ptr(g), _ptr(u), _ptr(out), g.numel()))
    return out


def moe_reduce(d: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """x += sum_s w[s] * d[s] in place (shaders/moe_reduce_f32.comp)."""
    check(lib().styx_moe_reduce(ctx(_dev(x)).handle, _stream(), _ptr(d), _ptr(w), _ptr(x), x.numel(), w.numel()))
    return x


def gather_slabs(srcs, src_bytes, arenas, dst_bytes, ids: torch.Tensor, layer: int, k: int,
                 n_expert: Optional[int] = None) -> None:
    """shaders/gather_slabs_f32.comp: srcs may be HostBuffer tensors (GTT)."""
    if n_expert is None:
        n_expert = srcs[0].numel() // src_bytes[0]
    check(lib().styx_gather_slabs(ctx(_dev(ids)).handle, _stream(), *[_ptr(s) for s in srcs], *src_bytes,
                                  *[_ptr(a) for a in arenas], *dst_bytes, _ptr(ids), n_expert, layer, k))


def gather_slabs_async(srcs, src_bytes, arenas, dst_bytes, host_ids, layer: int, k: int, stream=None,
                       n_expert: Optional[int] = None) -> None:
    if n_expert is None:
        n_expert = srcs[0].numel() // src_bytes[0]
    ids = (C.c_int32 * len(host_ids))(*[int(v) for v in host_ids])
    check(lib().styx_gather_slabs_async(ctx(_dev(arenas[0])).handle, _stream(stream), *[_ptr(s) for s in srcs],
                                        *src_bytes, *[_ptr(a) for a in arenas], *dst_bytes, ids, n_expert, layer,
                                        k))


def synth_quant(qtype: int, nrows: int, ncols: int, seed: int, sigma: float, out: Optional[torch.Tensor] = None,
                device: Optional[int] = None) -> torch.Tensor:
    """Synthetic N(0, sigma) rows quantised on the device."""
    rb = row_bytes(qtype, ncols)
    if out is None:
        out = torch.empty(nrows * rb, dtype=torch.uint8, device=f"cuda:{device if device is not None else torch.cuda.current_device()}")
    check(lib().styx_synth_quant(ctx(_dev(out)).handle, _stream(), qtype, _ptr(out), nrows, ncols, seed, sigma))
    return out


def synth_f32(n: int, seed: int, offset: int, sigma: float, device: Optional[int] = None) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=f"cuda:{device if device is not None else torch.cuda.current_device()}")
    check(lib().styx_synth_f32(ctx(_dev(out)).handle, _stream(), _ptr(out), n, seed, offset, sigma))
    return out


# ------------------------------------------------------------ MoE block
@dataclass
class Experts:
    """One expert tensor and its placement (ExpMat, moe.rs:97-106).

    full: uint8 [E*slab] (device); hot: dense hot slabs or None; arena: the
    arena base or None (global slot = layer*k + s)."""
    qtype: int
    full: Optional[torch.Tensor]
    slab_bytes: int
    hot: Optional[torch.Tensor] = None
    arena: Optional[torch.Tensor] = None
    arena_slab_bytes: int = 0

    def struct(self) -> ExpertTensor:
        n_hot = self.hot.numel() // self.slab_bytes if self.hot is not None else 0
        n_arena = self.arena.numel() // self.arena_slab_bytes if self.arena is not None else 0
        return ExpertTensor(self.full.data_ptr() if self.full is not None else None,
                            self.hot.data_ptr() if self.hot is not None else None,
                            self.arena.data_ptr() if self.arena is not None else None,
                            self.slab_bytes, self.arena_slab_bytes, self.qtype, n_hot, n_arena)


@dataclass
class LayerWeights:
    """Per-layer MoE weights (Layer, moe.rs:108-144)."""
    ffn_norm: torch.Tensor          # f32[H]
    router: torch.Tensor            # f32[E][H]
    gate: Experts
    up: Experts
    down: Experts
    remap: Optional[torch.Tensor] = None   # i32/u32[E], -1 = SKIP
    pmap: Optional[torch.Tensor] = None

    def struct(self) -> MoeLayer:
        return MoeLayer(self.ffn_norm.data_ptr(), self.router.data_ptr(),
                        self.remap.data_ptr() if self.remap is not None else None,
                        self.pmap.data_ptr() if self.pmap is not None else None,
                        self.gate.struct(), self.up.struct(), self.down.struct())


@dataclass
class Dims:
    n_embd: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    norm_topk: bool = True
    rms_eps: float = 1e-6

    def struct(self) -> MoeDims:
        return MoeDims(self.n_embd, self.n_ff, self.n_expert, self.n_expert_used, int(self.norm_topk),
                       self.rms_eps)


class MoeBlock:
    """The MoE block of MoeModel::forward_token on one device.

    Holds the workspace; `forward` runs route, gate/up+SiLU and
    down+combine (3 kernels) and updates x in place."""

    def __init__(self, dims: Dims, device: int = 0):
        self.dims = dims
        self.device = device
        self._dims = dims.struct()
        n = C.c_uint64()
        check(lib().styx_moe_workspace_bytes(C.byref(self._dims), C.byref(n)))
        self.ws_bytes = n.value
        self.workspace = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=f"cuda:{device}")
        self.ctx = ctx(device)
        self._structs: dict[int, MoeLayer] = {}

    def forward(self, x: torch.Tensor, layer_w: LayerWeights, layer: int, ids: torch.Tensor,
                weights_out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        st = layer_w.struct()
        check(lib().styx_moe_block(self.ctx.handle, _stream(stream), C.byref(self._dims), C.byref(st), layer,
                                   _ptr(x), _ptr(ids), _ptr(weights_out), _ptr(self.workspace),
                                   self.ws_bytes))
        return x

    def forward_layers(self, x: torch.Tensor, layer_ws: list, first_layer: int, ids: torch.Tensor,
                       weights_out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """Consecutive layers first_layer.. of one token (styx_moe_blocks):
        the same as forward() per layer in order; when every layer takes the
        single kernel, up to 80 of them run in one launch."""
        arr = (MoeLayer * len(layer_ws))(*[lw.struct() for lw in layer_ws])
        check(lib().styx_moe_blocks(self.ctx.handle, _stream(stream), C.byref(self._dims), arr, len(layer_ws),
                                    first_layer, _ptr(x), _ptr(ids), _ptr(weights_out), _ptr(self.workspace),
                                    self.ws_bytes))
        return x

    def forward_ep(self, x: torch.Tensor, layer_w: LayerWeights, layer: int, ids: torch.Tensor,
                   partial: torch.Tensor, weights_out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """Expert-parallel half of the block: partial[s, r] = w[s] * d[s][r]
        for the slots whose experts this rank holds (0 elsewhere); x is not
        updated.  Sum `partial` over the ranks, then `combine`."""
        st = layer_w.struct()
        check(lib().styx_moe_block_ep(self.ctx.handle, _stream(stream), C.byref(self._dims), C.byref(st), layer,
                                      _ptr(x), _ptr(ids), _ptr(weights_out), _ptr(partial), _ptr(self.workspace),
                                      self.ws_bytes))
        return partial

    def combine(self, partial: torch.Tensor, x: torch.Tensor, stream=None) -> torch.Tensor:
        """x += the slot-ordered sum of the (rank-summed) partials."""
        check(lib().styx_moe_combine(self.ctx.handle, _stream(stream), _ptr(partial), _ptr(x), self.dims.n_embd,
                                     self.dims.n_expert_used))
        return x

    def view(self, which: int, n: int) -> torch.Tensor:
        """xnorm (0), logits (1), h (2), weights (3) of the last forward."""
        p = C.c_void_p()
        check(lib().styx_moe_workspace_view(C.byref(self._dims), _ptr(self.workspace), which, C.byref(p)))
        off = p.value - self.workspace.data_ptr()
        return self.workspace[off: off + 4 * n].view(torch.float32)


class EpComm:
    """styx_ep: the cross-rank sum of the expert-parallel slot buffer and the
    combine into x, as one kernel over NVLink peer memory (no library
    collective).  Every rank opens one, the ranks exchange handles (any host
    channel: `connect_with` uses torch.distributed), then every rank calls
    `combine` (or `moe_block`) once per layer in the same order."""

    HANDLE_BYTES = 64

    def __init__(self, rank: int, world: int, k: int, n_embd: int, device: int = 0):
        self.ctx = ctx(device)
        self.handle = C.c_void_p()
        self._local = (C.c_uint8 * self.HANDLE_BYTES)()
        check(lib().styx_ep_open(self.ctx.handle, rank, world, k, n_embd, C.byref(self.handle), self._local))
        self.rank, self.world = rank, world

    def local_handle(self) -> bytes:
        return bytes(self._local)

    def connect(self, handles) -> None:
        """handles: every rank's local_handle(), in rank order."""
        buf = b"".join(handles)
        assert len(buf) == self.world * self.HANDLE_BYTES
        check(lib().styx_ep_connect(self.handle, buf))

    def connect_with(self, dist) -> None:
        """Exchanges the handles over a torch.distributed process group."""
        got = [None] * self.world
        dist.all_gather_object(got, self.local_handle())
        self.connect(got)

    def combine(self, partial: torch.Tensor, x: torch.Tensor, stream=None) -> torch.Tensor:
        """x += the slot-ordered sum over the ranks of their partials."""
        check(lib().styx_ep_combine(self.ctx.handle, self.handle, _stream(stream), _ptr(partial), _ptr(x)))
        return x

    def moe_block(self, blk: "MoeBlock", x: torch.Tensor, layer_w: LayerWeights, layer: int, ids: torch.Tensor,
                  weights_out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """The whole expert-parallel MoE block (styx_ep_moe_block): x ends
        as the single-device block leaves it.  Where the single kernel fits,
        the exchange is its epilogue (one launch per layer)."""
        st = layer_w.struct()
        check(lib().styx_ep_moe_block(blk.ctx.handle, self.handle, _stream(stream), C.byref(blk._dims), C.byref(st),
                                      layer, _ptr(x), _ptr(ids), _ptr(weights_out), _ptr(blk.workspace),
                                      blk.ws_bytes))
        return x

    def close(self) -> None:
        if self.handle:
            check(lib().styx_ep_close(self.handle))
            self.handle = C.c_void_p()


class MoeBatch:
    """The MoE block of a batch of up to 64 tokens of one layer
    (styx_moe_block_batch: grouped expert GEMMs on the tensor cores)."""

    def __init__(self, dims: Dims, n_tokens: int, device: int = 0):
        self.dims, self.n_tokens, self.device = dims, n_tokens, device
        self._dims = dims.struct()
        n = C.c_uint64()
        check(lib().styx_moe_batch_workspace_bytes(C.byref(self._dims), n_tokens, C.byref(n)))
        self.ws_bytes = n.value
        self.workspace = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=f"cuda:{device}")
        self.ctx = ctx(device)

    def forward(self, x: torch.Tensor, layer_w: LayerWeights, ids: torch.Tensor, weights_out: torch.Tensor,
                stream=None) -> torch.Tensor:
        """x: f32[n_tokens][n_embd] (in place); ids: int32[n_tokens * 64];
        weights_out: f32[n_tokens * k]."""
        st = layer_w.struct()
        check(lib().styx_moe_block_batch(self.ctx.handle, _stream(stream), C.byref(self._dims), C.byref(st),
                                         self.n_tokens, _ptr(x), _ptr(ids), _ptr(weights_out),
                                         _ptr(self.workspace), self.ws_bytes))
        return x


# ---------------------------------------------------------------- residency
def expert_budget(device_vram: int, headroom: int = 1024 << 20, pinned: int = 0, kv_max: int = 0,
                  arena: int = 0, explicit: Optional[int] = None, all_vram: bool = False) -> int:
    """MoeModel::load's expert VRAM budget (moe.rs:741-753), in bytes."""
    return lib().styx_expert_budget(device_vram, headroom, pinned, kv_max, arena, int(explicit is not None),
                                    explicit or 0, int(all_vram))


def arena_bytes(n_layers: int, k: int, max_slab: tuple) -> int:
    """The gather arena's size (moe.rs:727-740)."""
    arr = (C.c_uint64 * 3)(*max_slab)
    return lib().styx_arena_bytes(n_layers, k, arr)


class Residency:
    """Expert placement of MoeModel (moe.rs:692-813, 984-995, 1450-1521,
    2169-2213): popularity pinning, the per-layer remap tables the kernels
    read, online repin decisions, HUD counts and the prefetch plan.  Host
    logic only (libstyx_moe.so, C++); `apply_swaps` applies a repin on the
    device with styx_copy, as the reference does with copy_region."""

    def __init__(self, n_layers: int, n_expert: int, k: int, cost_per_expert: int):
        import numpy as np
        self._np = np
        self.n_layers, self.n_expert, self.k = n_layers, n_expert, k
        h = C.c_void_p()
        check(lib().styx_residency_create(n_layers, n_expert, k, cost_per_expert, C.byref(h)))
        self.handle = h
        self._destroy = lib().styx_residency_destroy   # still bound at interpreter exit

    def __del__(self):
        if getattr(self, "handle", None):
            self._destroy(self.handle)
            self.handle = None

    def _ids(self, ids):
        a = self._np.ascontiguousarray(ids, dtype=self._np.int32).reshape(-1)
        assert a.size >= self.n_layers * IDS_PER_LAYER, "ids: n_layers x 64 int32"
        return a

    def pin(self, layer, expert, hits, budget: int) -> int:
        np = self._np
        la = np.ascontiguousarray(layer, np.int32)
        ea = np.ascontiguousarray(expert, np.int32)
        ha = np.ascontiguousarray(hits, np.uint64)
        n = C.c_int()
        check(lib().styx_residency_pin(self.handle, la.ctypes.data, ea.ctypes.data, ha.ctypes.data, la.size,
                                       budget, C.byref(n)))
        return n.value

    def pin_csv(self, text: str, budget: int) -> int:
        raw = text.encode()
        n = C.c_int()
        check(lib().styx_residency_pin_csv(self.handle, raw, len(raw), budget, C.byref(n)))
        return n.value

    def layer(self, layer: int):
        """(remap u32[E], slot_experts u32[n_slots]) of one layer."""
        np = self._np
        remap = np.empty(self.n_expert, np.uint32)
        slots = np.empty(self.n_expert, np.uint32)
        n = C.c_int()
        check(lib().styx_residency_layer(self.handle, layer, remap.ctypes.data, slots.ctypes.data, C.byref(n)))
        return remap, slots[: n.value].copy()

    def hits(self, layer: int):
        h = self._np.empty(self.n_expert, self._np.uint64)
        check(lib().styx_residency_hits(self.handle, layer, h.ctypes.data))
        return h

    def maybe_repin(self, ids, n_past: int, interval: int, max_per_layer: int = 2):
        """MoeModel::maybe_repin: list of (layer, slot, old_expert, new_expert)."""
        a = self._ids(ids)
        cap = self.n_layers * max(max_per_layer, 0)
        buf = (_lib.RepinSwap * max(cap, 1))()
        n = C.c_int()
        check(lib().styx_residency_maybe_repin(self.handle, a.ctypes.data, n_past, interval, max_per_layer, buf,
                                               cap, C.byref(n)))
        return [(buf[i].layer, buf[i].slot, buf[i].old_expert, buf[i].new_expert) for i in range(n.value)]

    def hot_cold(self, ids):
        np = self._np
        a = self._ids(ids)
        hot = np.empty(self.n_layers, np.uint32)
        cold = np.empty(self.n_layers, np.uint32)
        check(lib().styx_residency_hot_cold(self.handle, a.ctypes.data, hot.ctypes.data, cold.ctypes.data))
        return hot, cold

    def prefetch_plan(self, ids):
        """(pmap u32[n_layers, E], pf_ids int32[n_layers, 64]) for the next token."""
        np = self._np
        a = self._ids(ids)
        pmap = np.empty((self.n_layers, self.n_expert), np.uint32)
        pf = np.full((self.n_layers, IDS_PER_LAYER), -1, np.int32)
        check(lib().styx_residency_prefetch_plan(self.handle, a.ctypes.data, pmap.ctypes.data, pf.ctypes.data))
        return pmap, pf

    def apply_swaps(self, swaps, layers: list, remaps: list, stream=None) -> None:
        """Apply repin swaps on the device (moe.rs:1482-1504): for each swap
        copy the new expert's slab of the full gate/up/down tensors into its
        hot slot (styx_copy), then upload each touched layer's remap table.
        layers[l]: LayerWeights with full and hot tensors; remaps[l]: the
        device remap tensor (int32/uint32[E]) the kernels read."""
        cx = ctx(layers[0].gate.full.device.index).handle
        touched = set()
        for (l, slot, _old, new) in swaps:
            lw = layers[l]
            for ex in (lw.gate, lw.up, lw.down):
                check(lib().styx_copy(cx, _ptr(ex.full), new * ex.slab_bytes, _ptr(ex.hot), slot * ex.slab_bytes,
                                      ex.slab_bytes, _stream(stream)))
            touched.add(l)
        for l in sorted(touched):
            remap, _ = self.layer(l)
            host = torch.from_numpy(remap.view(self._np.int32).copy())
            check(lib().styx_upload(cx, _ptr(remaps[l]), 0, C.c_void_p(host.data_ptr()), host.numel() * 4,
                                    _stream(stream)))
            if stream is None:
                torch.cuda.synchronize(remaps[l].device)


# ------------------------------------------------------------ attention half of a decode layer
# include/styx_attn.h: the part of forward_token before each MoE block
# (crates/model/src/moe.rs:1845-1972).

def mul_mat_vec(qtype: int, a: torch.Tensor, nrows: int, ncols: int, x: torch.Tensor,
                y: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """y = W x for a quantised row-major W (rec_matvec_b, moe.rs:1523-1551)."""
    if y is None:
        y = torch.empty(nrows, dtype=torch.float32, device=x.device)
    check(lib().styx_mul_mat_vec(ctx(_dev(x)).handle, _stream(stream), qtype, _ptr(a), nrows, ncols, _ptr(x),
                                 _ptr(y)))
    return y


def mul_mat_vec_add(qtype: int, a: torch.Tensor, nrows: int, ncols: int, x: torch.Tensor, y: torch.Tensor,
                    stream=None) -> torch.Tensor:
    """y += W x (the o projection with the residual add fused)."""
    check(lib().styx_mul_mat_vec_add(ctx(_dev(x)).handle, _stream(stream), qtype, _ptr(a), nrows, ncols, _ptr(x),
                                     _ptr(y)))
    return y


def add_f32(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """add_flat_f32: out = a + b (out may be a)."""
    if out is None:
        out = torch.empty_like(a)
    check(lib().styx_add_f32(ctx(_dev(a)).handle, _stream(stream), _ptr(a), _ptr(b), _ptr(out), a.numel()))
    return out


def qk_norm_rope_kv(q: torch.Tensor, k: torch.Tensor, v: Optional[torch.Tensor], q_norm, k_norm, eps: float,
                    n_heads: int, n_kv: int, head_dim: int, freq_base: float, pos: torch.Tensor,
                    kcache: Optional[torch.Tensor] = None, vcache: Optional[torch.Tensor] = None,
                    n_ctx: int = 0, n_tokens: int = 1, stream=None) -> None:
    """Per-head q/k RMSNorm, NEOX RoPE at pos (device int32[n_tokens]) and the
    K / V cache rows, in place (moe.rs:1880-1945)."""
    check(lib().styx_qk_norm_rope_kv(ctx(_dev(pos)).handle, _stream(stream), _ptr(q), _ptr(k), _ptr(v),
                                     _ptr(q_norm), _ptr(k_norm), eps, n_heads, n_kv, head_dim, n_tokens, freq_base,
                                     _ptr(pos), _ptr(kcache), _ptr(vcache), n_ctx))


def rope_neox(x: torch.Tensor, head_dim: int, n_heads: int, n_tokens: int, freq_base: float, pos: torch.Tensor,
              stream=None) -> torch.Tensor:
    """rope_neox_f32 in place over x f32[n_tokens][n_heads][head_dim]."""
    check(lib().styx_rope_neox(ctx(_dev(x)).handle, _stream(stream), _ptr(x), head_dim, n_heads, n_tokens,
                               freq_base, _ptr(pos)))
    return x


def attn_workspace_bytes(n_heads: int, head_dim: int) -> int:
    v = C.c_uint64()
    check(lib().styx_attn_workspace_bytes(n_heads, head_dim, C.byref(v)))
    return v.value


def attn_decode(q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, n_t: int, head_dim: int,
                kv_dim: int, gqa: int, scale: float, out: Optional[torch.Tensor] = None,
                workspace: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """attn_decode_f32: out[h] = softmax(scale q[h].K[:n_t, h/gqa]) V[:n_t, h/gqa]."""
    n_heads = gqa * (kv_dim // head_dim)
    if out is None:
        out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    nb = attn_workspace_bytes(n_heads, head_dim)
    if workspace is None:
        workspace = torch.empty(nb, dtype=torch.uint8, device=q.device)
    check(lib().styx_attn_decode(ctx(_dev(q)).handle, _stream(stream), _ptr(q), _ptr(kcache), _ptr(vcache),
                                 _ptr(out), n_t, head_dim, kv_dim, gqa, scale, _ptr(workspace), workspace.numel()))
    return out


@dataclass
class DenseWeight:
    qtype: int
    data: torch.Tensor     # raw blocks, row-major

    def struct(self) -> _lib.DenseTensor:
        return _lib.DenseTensor(self.data.data_ptr(), self.qtype)


@dataclass
class AttnWeights:
    attn_norm: torch.Tensor
    wq: DenseWeight
    wk: DenseWeight
    wv: DenseWeight
    wo: DenseWeight
    q_norm: Optional[torch.Tensor] = None
    k_norm: Optional[torch.Tensor] = None

    def struct(self) -> _lib.AttnLayer:
        return _lib.AttnLayer(self.attn_norm.data_ptr(), self.wq.struct(), self.wk.struct(), self.wv.struct(),
                              self.wo.struct(), self.q_norm.data_ptr() if self.q_norm is not None else None,
                              self.k_norm.data_ptr() if self.k_norm is not None else None)


class AttnBlock:
    """One layer's attention half (styx_attn_block) with its workspace."""

    def __init__(self, n_embd: int, n_heads: int, n_kv_heads: int, head_dim: int, qk_norm: bool,
                 rms_eps: float, rope_base: float, device: int = 0):
        self.dims = _lib.AttnDims(n_embd, n_heads, n_kv_heads, head_dim, int(qk_norm), rms_eps, rope_base)
        self.ctx = ctx(device)
        v = C.c_uint64()
        check(lib().styx_attn_block_workspace_bytes(C.byref(self.dims), C.byref(v)))
        self.ws_bytes = v.value
        self.workspace = torch.empty(self.ws_bytes, dtype=torch.uint8, device=f"cuda:{device}")
        self.init_workspace()

    def init_workspace(self, stream=None) -> None:
        check(lib().styx_attn_block_workspace_init(self.ctx.handle, _stream(stream), _ptr(self.workspace),
                                                   self.ws_bytes))

    def last_path(self) -> int:
        """1: the last forward ran as one kernel, 2: as seven."""
        return self.ctx.get_option(_lib.OPT_ATTN_LAST_PATH)

    def forward(self, x: torch.Tensor, w: AttnWeights, pos: int, pos_dev: torch.Tensor, kcache: torch.Tensor,
                vcache: torch.Tensor, n_ctx: int, stream=None) -> torch.Tensor:
        st = w.struct()
        check(lib().styx_attn_block(self.ctx.handle, _stream(stream), C.byref(self.dims), C.byref(st), _ptr(x), pos,
                                    _ptr(pos_dev), _ptr(kcache), _ptr(vcache), n_ctx, _ptr(self.workspace),
                                    self.ws_bytes))
        return x


def get_rows(qtype: int, w: torch.Tensor, nrows: int, ncols: int, rows: torch.Tensor,
             out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Dequantised rows of a quantised matrix (the token embedding)."""
    n = rows.numel()
    if out is None:
        out = torch.empty(n, ncols, dtype=torch.float32, device=rows.device)
    check(lib().styx_get_rows(ctx(_dev(rows)).handle, _stream(stream), qtype, _ptr(w), nrows, ncols, _ptr(rows), n,
                              _ptr(out)))
    return out


def argmax_f32(x: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Greedy pick: the last index of the maximum under IEEE total order."""
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=x.device)
    check(lib().styx_argmax_f32(ctx(_dev(x)).handle, _stream(stream), _ptr(x), x.numel(), _ptr(out)))
    return out
