"""Tensor parallelism for the Q4_0 decode step: the load-time sharding hook and
the per-layer all-gather.

Across G GPUs of one box the path is split only where it shards by itself:

* every Q4_0 linear is column-sharded along N (its output features). A GGML
  Q4_0 row is K/32 whole 18-byte blocks, so rank r's rows [r N/G, (r+1) N/G)
  are one contiguous byte slice of the blob -- no re-quantisation, the same
  bytes `_quantized_to` (torch_c/src/quant.rs:384-405) would move;
* attention is split by KV-head group: rank r owns KV heads
  [r Hkv/G, (r+1) Hkv/G) and the Hq/Hkv query heads that read each of them
  (the GQA map of aten.rs:17106-17130), so no exchange is needed inside
  attention. The fused q/k/v weight is sliced per section (q rows, k rows,
  v rows) so the local projection has the same [q | k | v] layout;
* after each sharded linear one NCCL all-gather over NVLink/NVSwitch
  rebuilds the full activation row on every rank (4 per layer: attention
  output, o_proj, SiLU(gate)*up, down_proj; plus the lm_head logits), and the
  replicated parts (residual, RMSNorm, argmax) run on every rank -- the
  "colwise" plan, whose token stream is the one-GPU stream bit for bit;
* or ("rowwise", transformers' colwise/rowwise plan) o_proj and down_proj
  are row-parallel: rank r keeps input features [r K/G, (r+1) K/G) of every
  row (its own heads' attention output, its own SiLU*up columns), so the
  attention output and SiLU*up stay local, and each of the two linears ends
  in an all-reduce of f32 partials fused into its own kernel: 2 exchanges a
  layer instead of 4, no exchange launches.

The reference has no multi-GPU path; the hook sits where its model-load path
adopts quantised weights (torchnative/python/torchnative/quant/hf.py:340 and
quant/__init__.py:183-237).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N

P = ctypes.c_void_p


def q4_row_bytes(k: int) -> int:
    if k % 32 != 0:
        raise ValueError(f"a q4_0 row is whole 32-element blocks, got in_features {k}")
    return k // 32 * 18


def row_slice(blob: torch.Tensor, n: int, k: int, start: int, stop: int) -> torch.Tensor:
    """Rows [start, stop) of an [n, k] Q4_0 blob (uint8, flat) as a new
    contiguous blob."""
    rb = q4_row_bytes(k)
    if blob.numel() != n * rb:
        raise ValueError(f"q4_0 blob of {blob.numel()} bytes is not [{n}, {k}] ({n * rb} bytes)")
    if not 0 <= start <= stop <= n:
        raise ValueError(f"row range [{start}, {stop}) outside [0, {n})")
    return blob[start * rb:stop * rb].clone()


def _split(n: int, world: int, what: str) -> int:
    if n % world != 0:
        raise ValueError(f"{what} ({n}) does not divide by the tensor-parallel size {world}")
    return n // world


def shard_rows(blob: torch.Tensor, n: int, k: int, rank: int, world: int) -> torch.Tensor:
    """Column-sharded linear: rank r's output features [r n/G, (r+1) n/G)."""
    c = _split(n, world, "out_features")
    return row_slice(blob, n, k, rank * c, (rank + 1) * c)


def shard_qkv(blob: torch.Tensor, heads: int, kv_heads: int, head_dim: int, k: int, rank: int,
              world: int) -> torch.Tensor:
    """The fused [q | k | v] projection of rank r's KV-head group: query heads
    [r Hq/G, (r+1) Hq/G), key and value heads [r Hkv/G, (r+1) Hkv/G)."""
    hq, hkv = _split(heads, world, "query heads"), _split(kv_heads, world, "key/value heads")
    n = (heads + 2 * kv_heads) * head_dim
    q0 = rank * hq * head_dim
    k0 = heads * head_dim + rank * hkv * head_dim
    v0 = (heads + kv_heads) * head_dim + rank * hkv * head_dim
    return torch.cat([row_slice(blob, n, k, q0, q0 + hq * head_dim),
                      row_slice(blob, n, k, k0, k0 + hkv * head_dim),
                      row_slice(blob, n, k, v0, v0 + hkv * head_dim)])


def shard_cols(blob: torch.Tensor, n: int, k: int, rank: int, world: int) -> torch.Tensor:
    """Row-parallel linear: rank r's input features [r k/G, (r+1) k/G) of every
    output row -- whole Q4_0 blocks of each row (k/G a multiple of 32), cut out
    of the blob as bytes and packed as an [n, k/G] blob."""
    rb = q4_row_bytes(k)
    c = _split(k // 32, world, "in_features / 32")
    if blob.numel() != n * rb:
        raise ValueError(f"q4_0 blob of {blob.numel()} bytes is not [{n}, {k}] ({n * rb} bytes)")
    return blob.view(n, k // 32, 18)[:, rank * c:(rank + 1) * c].reshape(-1).contiguous()


def shard_gate_up_pairs(blob: torch.Tensor, inter: int, k: int, rank: int, world: int) -> torch.Tensor:
    """gate/up interleaved row by row (2i = gate_i, 2i+1 = up_i): rank r's
    pairs [r I/G, (r+1) I/G) are rows [2 r I/G, 2 (r+1) I/G)."""
    c = _split(inter, world, "intermediate size")
    return row_slice(blob, 2 * inter, k, 2 * rank * c, 2 * (rank + 1) * c)


class PeerLost(TimeoutError):
    """A rank of the tensor-parallel group did not take part in a collective:
    it left, or did not arrive within the process group's timeout."""


_LOST_SIGNS = ("timed out", "timeout", "connection closed", "connection reset", "broken pipe", "peer")


@dataclass
class TPGroup:
    """One tensor-parallel group: this process's rank, the group size and the
    torch.distributed process group (NCCL on GPUs, gloo in CPU tests)."""
    rank: int
    world: int
    group: object = None

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        """out = concatenation over ranks of inp (rank-major). NCCL: one
        all_gather_into_tensor on the current stream (captured with the step
        inside a CUDA-graph capture); gloo (CPU tests): the list form."""
        import torch.distributed as dist

        try:
            if dist.get_backend(self.group) == "gloo":
                parts = list(out.view(self.world, -1).unbind(0))
                dist.all_gather(parts, inp.reshape(-1), group=self.group)
                return
            dist.all_gather_into_tensor(out, inp, group=self.group)
        except RuntimeError as e:
            if any(sign in str(e).lower() for sign in _LOST_SIGNS):
                raise PeerLost(f"tensor-parallel all-gather, rank {self.rank} of {self.world}: a peer rank did not "
                               f"take part ({e})") from e
            raise


def gather_rows(tp: TPGroup, local: torch.Tensor, full: torch.Tensor, scratch: torch.Tensor | None,
                stream) -> None:
    """full[b] = concat over ranks of rank r's local[b] ([rows, c] each, 16-bit
    elements): one all-gather, plus the layout step when rows > 1."""
    rows, c = local.shape
    if rows == 1:
        tp.all_gather(full.view(-1), local.view(-1))
        return
    buf = scratch.view(-1)[:tp.world * rows * c]
    tp.all_gather(buf, local.reshape(-1))
    N.check(N.lib().tn_tp_unshard(P(buf.data_ptr()), P(full.data_ptr()), tp.world, rows, c, stream))


class _DevicePointer:
    """A raw device pointer presented through the CUDA array interface, so
    torch can view memory this library allocated (16-bit elements as int16)."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerExchange:
    """This rank's exchange region and its peers' (CUDA IPC, plain peer
    mappings), for tn_tp_allgather. Buffers handed out by `buffer()` are the
    gather destinations: every rank writes its slice of them directly."""

    def __init__(self, tp: TPGroup, nbytes: int, device):
        import torch.distributed as dist

        self.tp, self.dev = tp, torch.device(device)
        lib = N.lib()
        handle = (ctypes.c_uint8 * 64)()
        base = ctypes.c_void_p()
        N.check(lib.tn_tp_region_alloc(nbytes, ctypes.byref(base), handle))
        self.base = base.value
        self.nbytes = nbytes
        self.data_off = int(lib.tn_tp_region_data_offset())
        handles = [None] * tp.world
        dist.all_gather_object(handles, bytes(handle), group=tp.group)
        self.bases = (ctypes.c_void_p * tp.world)()
        self._opened = []
        for g in range(tp.world):
            if g == tp.rank:
                self.bases[g] = self.base
                continue
            h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[g])
            peer = ctypes.c_void_p()
            N.check(lib.tn_tp_region_open(h, ctypes.byref(peer)))
            self.bases[g] = peer.value
            self._opened.append(peer.value)
        self._next = 0

    def buffer(self, rows: int, cols: int, dtype=torch.bfloat16) -> tuple[torch.Tensor, int]:
        """A [rows, cols] 16-bit gather destination in this rank's region and
        its byte offset in the data area (256-byte aligned)."""
        off = self._next
        size = rows * cols * 2
        if off + size > self.nbytes:
            raise ValueError("exchange region too small")
        self._next = (off + size + 255) // 256 * 256
        t = torch.as_tensor(_DevicePointer(self.base + self.data_off + off, rows * cols), device=self.dev)
        return t.view(dtype).view(rows, cols), off

    def allgather(self, local: torch.Tensor, dst_off: int, full_cols: int, slot: int, stream) -> None:
        """Gather `slot` of this step: local [rows, c] -> every rank's [rows, full_cols] at dst_off."""
        rows, c = local.shape
        N.check(N.lib().tn_tp_allgather(self.bases, self.tp.rank, self.tp.world, P(local.data_ptr()),
                                        local.stride(0), rows, c, dst_off, full_cols, slot, stream))

    def reserve(self, nbytes: int) -> int:
        """nbytes of this rank's data area (256-byte aligned) with no tensor
        view: the row-parallel reductions' f32 partials."""
        off = self._next
        if off + nbytes > self.nbytes:
            raise ValueError("exchange region too small")
        self._next = (off + nbytes + 255) // 256 * 256
        return off

    def reduce_link(self, slot: int, partial_off: int, cols: int) -> "N.TpLink":
        """A tn_tp_link for a row-parallel GEMV with its all-reduce fused in:
        reduction `slot` of the step, its tagged f32 partials (8-byte words)
        at partial_off laid out [rows][world * cols]."""
        ln = N.TpLink()
        ln.world, ln.rank = self.tp.world, self.tp.rank
        for g in range(self.tp.world):
            ln.bases[g] = self.bases[g]
        ln.dst_offset, ln.dst_row_stride, ln.slot, ln.wait_slot, ln.reduce = (partial_off, self.tp.world * cols,
                                                                              slot, -1, 1)
        return ln

    def link(self, slot: int = -1, dst_off: int = 0, full_cols: int = 0, wait_slot: int = -1) -> "N.TpLink":
        """A tn_tp_link for a GEMV that feeds gather `slot` (its output scattered
        into every rank's buffer at dst_off) and/or reads gather `wait_slot`."""
        ln = N.TpLink()
        ln.world, ln.rank = self.tp.world, self.tp.rank
        for g in range(self.tp.world):
            ln.bases[g] = self.bases[g]
        ln.dst_offset, ln.dst_row_stride, ln.slot, ln.wait_slot = dst_off, full_cols, slot, wait_slot
        return ln

    def step_end(self, stream) -> None:
        N.check(N.lib().tn_tp_step_end(P(self.base), stream))

    def close(self) -> None:
        """After a barrier that no rank passes with a gather in flight."""
        lib = N.lib()
        for p in self._opened:
            lib.tn_tp_region_close(P(p))
        self._opened = []
        if self.base:
            lib.tn_tp_region_free(P(self.base))
            self.base = 0
