"""Symmetric device buffers and peer-memory collectives for one-process-per-GPU tensor parallelism.

`TPComm` owns, per rank, buffers allocated with cudaMalloc and exported through CUDA IPC; every
rank maps every peer's buffer, so the kernels in csrc/comm.cu can load from and store to other
GPUs over NVLink / NVSwitch. torch.distributed (any backend) is used only to exchange the IPC
handles at set-up. Device-side waits are bounded; `check()` raises if one expired.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..ops.kernels import _count
from ..ops.native import check_errors, err_word, lib

MAX_RANKS = 8


@dataclass
class SymTensor:
    """A symmetric buffer: the local tensor and every rank's base pointer (index = rank)."""

    local: torch.Tensor
    ptrs: List[int]

    def view_ptrs(self, offset_elems: int) -> List[int]:
        es = self.local.element_size()
        return [p + offset_elems * es for p in self.ptrs]


@dataclass
class BarrierChannel:
    """Flags of one barrier: slots [0, 8) written by the ranks, slot 8 the local epoch counter
    (kept on the device, so barriers can be captured into CUDA graphs and replayed)."""

    flags: SymTensor


class TPComm:
    def __init__(self, group: Optional["dist.ProcessGroup"] = None, device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.world > MAX_RANKS:
            raise ValueError(f"peer-memory TP supports at most {MAX_RANKS} ranks")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self._owned: List[int] = []
        self._opened: List[int] = []
        self.err = err_word(self.device)
        self._default = self.channel()

    def channel(self) -> "BarrierChannel":
        """An independent barrier (own flags and epoch), for work issued on its own stream."""
        return BarrierChannel(self.empty((2 * MAX_RANKS,), torch.int32))

    # ------------------------------------------------------------------ buffers
    def empty(self, shape: Sequence[int], dtype: torch.dtype) -> SymTensor:
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = max(n * torch.empty((), dtype=dtype).element_size(), 16)
        nbytes = (nbytes + 255) // 256 * 256
        with torch.cuda.device(self.device):
            ptr, handle = lib().ipc_alloc(nbytes)
        self._owned.append(ptr)
        handles: List[bytes] = [None] * self.world  # type: ignore
        if self.world > 1:
            dist.all_gather_object(handles, handle, group=self.group)
        else:
            handles = [handle]
        ptrs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(ptr)
                else:
                    p = lib().ipc_open(h)
                    self._opened.append(p)
                    ptrs.append(p)
        t = lib().tensor_from_ptr(ptr, [int(s) for s in shape], dtype, self.device.index)
        return SymTensor(t, ptrs)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib().ipc_close(p)
            for p in self._owned:
                lib().ipc_free(p)
        self._opened, self._owned = [], []

    # ------------------------------------------------------------------ collectives
    def barrier(self, ch: Optional["BarrierChannel"] = None) -> None:
        """Device-side barrier across the group on the current stream (bounded wait). Barriers
        of one channel must be issued in the same order on every rank."""
        if self.world == 1:
            return
        ch = ch or self._default
        _count()
        lib().tp_barrier(ch.flags.ptrs, self.rank, self.err)

    def sp_row(self, M: int, D: int, rows_per_rank: int, *, tok=None, src: Optional[Tuple[List[int], List[int]]] = None,
               bias=None, gamma=None, resid=None, resid_tok: bool = True, resid2=None,
               out=None, out_tok: bool = True, aux=None, aux_mode: int = 0, x=None, copy_out=None,
               ln_w=None, ln_b=None, eps: float = 1e-6, rms: bool = False, ag: Optional[SymTensor] = None,
               ag_scale: Optional[SymTensor] = None, ag_sf: Optional[SymTensor] = None, ag_push: bool = False) -> None:
        """Owner-side row kernel of the sequence-parallel layout (csrc/tp_sp.cu): finish the
        reduce-scatter of the partial rows `src` = (base pointers, row offsets), one per rank (or
        load x[tok]) on the rows this rank owns, then LayerNorm and all-gather the normalised
        rows into every rank's `ag` (e4m3 + row scales when ag_scale; NVFP4 -- packed e2m1 rows,
        row scales and blocked block scales -- when ag_sf is given too)."""
        _count()
        mode = 0 if ag_scale is None else (2 if ag_sf is not None else 1)
        # ag_push (contiguous rows only): the row kernel writes the gathered rows locally and a
        # bulk push with coalesced 16-byte peer stores sends them to the other ranks
        push = ag_push and tok is None and ag is not None and ln_w is not None and self.world > 1
        lib().sp_row(M, tok, rows_per_rank, self.rank, self.world, D, list(src[0]) if src else [],
                     list(src[1]) if src else [], bias, gamma, resid, resid_tok, resid2, out, out_tok, aux, aux_mode, x, copy_out,
                     ln_w, ln_b, float(eps), rms, mode, ag.ptrs if ag is not None else [],
                     (ag.local.stride(0) if ag is not None else 0), ag_scale.ptrs if mode else [],
                     ag_sf.ptrs if mode == 2 else [], push)
        if push:
            r0, r1 = min(M, self.rank * rows_per_rank), min(M, (self.rank + 1) * rows_per_rank)
            _count()
            lib().sp_push_ag(ag.ptrs, ag.local.stride(0) * ag.local.element_size(), r0, r1,
                             ag_scale.ptrs if mode else [], ag_sf.ptrs if mode == 2 else [],
                             D // 64 if mode == 2 else 0, self.rank)

    def push_rows(self, src: int, dst: List[int], tok: Optional[torch.Tensor], M: int, D: int,
                  rows_per_rank: int) -> None:
        """Copy every packed bf16 row i of `src` [M, D] whose owner (tok[i] // rows_per_rank, or
        i // rows_per_rank) is another rank into row i of that owner's `dst[owner]`
        (coalesced peer stores; the sending half of a reduce-scatter)."""
        if self.world == 1:
            return
        _count()
        lib().sp_push_rows(int(src), [int(p) for p in dst], tok, int(M), int(D), int(rows_per_rank), self.rank)

    def mean_f32(self, src: SymTensor, dst: torch.Tensor) -> None:
        _count()
        lib().tp_mean_f32(src.ptrs, dst)

    def check(self) -> None:
        check_errors(self.device)
