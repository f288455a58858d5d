"""Tensor-parallel exchange of the multi-GPU decode layer over NVLink peer memory.

`TPComm` owns, on every rank of a process group, four device buffers of its own allocation
(the fp32 O-projection partial, the bf16 layer output, the fused kernel's fp32 receive slots and
the flag words), exchanges their CUDA IPC handles once (torch.distributed is the plumbing:
all_gather_object) and maps the peers' buffers.  Two kernels use them:
  * `okc_tp_oproj_allreduce_residual` (set up when the O projection's K is given as
    `oproj_k`): the O projection fused with the exchange in one tcgen05 kernel, fp32 tile
    slices pushed into the owner rank's receive slots as each tile's accumulator completes,
    out = bf16(x + sum_r o_r @ wo_r^T) replicated on every rank;
  * `okc_tp_allreduce_residual`: out = bf16(x + sum_r partial_r) for a partial already in HBM
    (the expert-parallel MoE's shares), reading and writing the peers' memory directly.
They replace the NCCL all-reduce of the partial plus the residual add.  Every rank must
construct a TPComm and call it in the same order; it is CUDA-graph capturable (fixed buffers;
the per-CTA call epochs live on the device in `state`).
"""

from __future__ import annotations

import ctypes as C
import os

import torch
import torch.distributed as dist

from . import _lib, ops


_STATE_WORDS = 1024            # OKC_TP_STATE_WORDS
_EXCHANGE_FLAG_WORDS = 8192    # OKC_TP_EXCHANGE_FLAG_WORDS


class _DeviceBuffer:
    """A zero-filled cudaMalloc'd buffer (so its IPC handle maps exactly this buffer)."""

    def __init__(self, nbytes: int):
        self.ptr = C.c_void_p()
        _lib.check(_lib.load().okc_ipc_alloc(nbytes, C.byref(self.ptr)), "okc_ipc_alloc")
        self.nbytes = nbytes

    def handle(self) -> bytes:
        h = C.create_string_buffer(64)
        _lib.check(_lib.load().okc_ipc_handle(self.ptr, h), "okc_ipc_handle")
        return h.raw

    def free(self):
        if self.ptr:
            _lib.load().okc_ipc_free(self.ptr)
            self.ptr = C.c_void_p()


class _CudaArray:
    """__cuda_array_interface__ over memory this module owns (no copy, no ownership)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2}


def _from_ptr(ptr: int, nbytes: int, dtype, device) -> torch.Tensor:
    typestr, size = {torch.float32: ("<f4", 4), torch.bfloat16: ("<i2", 2), torch.int32: ("<i4", 4)}[dtype]
    t = torch.as_tensor(_CudaArray(ptr, nbytes // size, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class TPComm:
    """One exchange group: partial fp32 [T, H] -> out bf16 [T, H] on `world` ranks."""

    def __init__(self, T: int, H: int, group=None, device: int | None = None, oproj_k: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("TPComm needs 2..8 ranks")
        if (T * H) % 4:
            raise ValueError("T*H must be a multiple of 4")
        self.device = torch.cuda.current_device() if device is None else device
        self.T, self.H = T, H
        lib = _lib.load()
        self.oproj_k = None
        flag_words, recv_bytes = _EXCHANGE_FLAG_WORDS, 16  # exchange flags, then the fused kernel's
        if oproj_k is not None and os.environ.get("OKC_TP_FUSED", "1") != "0":
            rb, fw = C.c_size_t(), C.c_int()
            with torch.cuda.device(self.device):
                ok = lib.okc_tp_oproj_plan(T, H, oproj_k, self.world, C.byref(rb), C.byref(fw)) == 0
            agree = [None] * self.world  # every rank must take the same path
            dist.all_gather_object(agree, ok, group=group)
            if all(agree):
                self.oproj_k, recv_bytes = oproj_k, rb.value
                flag_words += fw.value
        with torch.cuda.device(self.device):
            self._part = _DeviceBuffer(T * H * 4)
            self._out = _DeviceBuffer(T * H * 2)
            self._flags = _DeviceBuffer(flag_words * 4)
            self._recv = _DeviceBuffer(recv_bytes)
            self.state = torch.zeros(_STATE_WORDS, dtype=torch.int32, device=f"cuda:{self.device}")
            mine = (self._part.handle(), self._out.handle(), self._flags.handle(), self._recv.handle())
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
            self._opened = []
            parts, outs, flags, recvs = [], [], [], []
            for q in range(self.world):
                if q == self.rank:
                    parts.append(self._part.ptr.value)
                    outs.append(self._out.ptr.value)
                    flags.append(self._flags.ptr.value)
                    recvs.append(self._recv.ptr.value)
                    continue
                ptrs = []
                for h in allh[q]:
                    p = C.c_void_p()
                    _lib.check(lib.okc_ipc_open(C.create_string_buffer(h, 64), C.byref(p)), "okc_ipc_open")
                    self._opened.append(p)
                    ptrs.append(p.value)
                parts.append(ptrs[0])
                outs.append(ptrs[1])
                flags.append(ptrs[2])
                recvs.append(ptrs[3])
            arr = C.c_void_p * self.world
            self._parts_arr = arr(*parts)
            self._outs_arr = arr(*outs)
            self._flags_arr = arr(*flags)
            self._flags_f_arr = arr(*[f + _EXCHANGE_FLAG_WORDS * 4 for f in flags])  # the fused kernel's words
            self._recv_arr = arr(*recvs)
            self.partial = _from_ptr(self._part.ptr.value, T * H * 4, torch.float32,
                                     f"cuda:{self.device}").view(T, H)
            self.out = _from_ptr(self._out.ptr.value, T * H * 2, torch.bfloat16,
                                 f"cuda:{self.device}").view(T, H)
            self._ws = ops.workspace(self.device, "tp", 4096)
        dist.barrier(group=group)

    def allreduce_residual(self, residual: torch.Tensor | None) -> torch.Tensor:
        """out = bf16(residual + sum over ranks of `self.partial`) on every rank (residual may
        be None); returns `self.out` (valid until the next call)."""
        if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != (self.T, self.H)
                                     or not residual.is_contiguous()):
            raise ValueError("residual must be a contiguous bf16 [T, H] tensor")
        lib = _lib.load()
        st = lib.okc_tp_allreduce_residual(self._parts_arr, self._outs_arr, self._flags_arr,
                                           None if residual is None else residual.data_ptr(),
                                           self.state.data_ptr(), self.rank, self.world, self.T * self.H,
                                           self._ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "okc_tp_allreduce_residual")
        return self.out

    def trace_stamps(self) -> torch.Tensor:
        """The phase trace of the last 4 calls of each kernel (int64 ns [2, 4, 16]: kernel 0 the
        exchange, 1 the fused O projection; slot = call epoch % 4), filled only when the
        library runs with OKC_TP_TRACE=1.  Synchronises."""
        torch.cuda.synchronize(self.device)
        return self._ws[256:256 + 2 * 64 * 8].view(torch.int64).view(2, 4, 16).cpu()

    @property
    def fused(self) -> bool:
        """True when `oproj_allreduce_residual` (the fused kernel) is set up on every rank."""
        return self.oproj_k is not None

    def oproj_allreduce_residual(self, x: torch.Tensor, w: torch.Tensor,
                                 residual: torch.Tensor | None) -> torch.Tensor:
        """out = bf16(residual + sum over ranks of x_r · w_r^T) on every rank, in one kernel:
        x bf16 [T, K] (this rank's attention output), w bf16 [H, K] (this rank's columns of the
        O weight), residual bf16 [T, H] or None.  Returns `self.out` (valid until the next call)."""
        if not self.fused:
            raise RuntimeError("the fused O projection was not set up (pass oproj_k; shape unsupported?)")
        K = self.oproj_k
        if (x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.shape != (self.T, K)
                or w.shape != (self.H, K) or not x.is_contiguous() or not w.is_contiguous()):
            raise ValueError(f"x must be bf16 [{self.T}, {K}] and w bf16 [{self.H}, {K}], both contiguous")
        if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != (self.T, self.H)
                                     or not residual.is_contiguous()):
            raise ValueError("residual must be a contiguous bf16 [T, H] tensor")
        st = _lib.load().okc_tp_oproj_allreduce_residual(
            x.data_ptr(), K, w.data_ptr(), K, self.T, self.H, K, self._recv_arr, self._outs_arr, self._flags_f_arr,
            None if residual is None else residual.data_ptr(), self.H, self.state.data_ptr(), self.rank, self.world,
            self._ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "okc_tp_oproj_allreduce_residual")
        return self.out

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (call on every rank, after a
        barrier, when no kernel that uses them is in flight)."""
        lib = _lib.load()
        for p in self._opened:
            lib.okc_ipc_close(p)
        self._opened = []
        for b in (self._part, self._out, self._flags, self._recv):
            b.free()


class ExpertParallelMoE:
    """Expert-parallel W4A16 MoE over the ranks of `group`.

    Rank r holds experts [expert_lo, expert_lo + E_local) of the bank (its slices of w13/w2 and
    their scales).  Routing is computed on every rank (bit-exact, so the ranks agree on every
    id); each rank runs its local experts for the pairs routed to them and leaves its fp32
    share of the weighted sum in the exchange buffer, and `okc_tp_allreduce_residual` sums the
    shares over NVLink (plus an optional residual) into the replicated bf16 output.  With the
    tokens replicated on every rank (tensor-parallel attention before the MoE) this is the
    all-to-all dispatch + combine with the dispatch already in place."""

    def __init__(self, router: torch.Tensor, w13, w13_sf, w13_gs, w2, w2_sf, w2_gs, expert_lo: int,
                 topk: int, group=None, renormalize: bool = True):
        self.router = router
        self.w13, self.w13_sf, self.w13_gs = w13, w13_sf, w13_gs
        self.w2, self.w2_sf, self.w2_gs = w2, w2_sf, w2_gs
        self.expert_lo, self.E_local = expert_lo, w13.shape[0]
        self.topk, self.group, self.renormalize = topk, group, renormalize
        self._comms: dict[int, TPComm] = {}
        self._gather: dict = {}

    def comm_for(self, tokens: int) -> TPComm:
        """The exchange group for `tokens` rows (created on first use: every rank together,
        outside graph capture)."""
        c = self._comms.get(tokens)
        if c is None:
            c = TPComm(tokens, self.w2.shape[1], group=self.group)
            self._comms[tokens] = c
        return c

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """bf16 [T, H] = (residual +) sum over the top-k experts of weight * expert(x)."""
        ids, wts = ops.moe_route(x, self.router, self.topk, self.renormalize)
        perm = ops.moe_permute(ids, self.expert_lo, self.E_local)
        comm = self.comm_for(x.shape[0])
        ops.moe_experts(x, ids, wts, perm, self.w13, self.w13_sf, self.w13_gs, self.w2, self.w2_sf, self.w2_gs,
                        self.expert_lo, out=comm.partial, out_fp32=True)
        return comm.allreduce_residual(residual)

    def forward_local(self, x: torch.Tensor) -> torch.Tensor:
        """Data-parallel tokens: each rank holds its own rows x_r [T, H] (the same T on every
        rank) and gets back bf16 [T, H] = the MoE of its rows.  Dispatch: the rows of all ranks
        are all-gathered into [W*T, H] (NCCL over NVLink; fixed sizes, so no host
        synchronisation and the call can be captured in a graph).  Each rank routes all W*T rows
        (bit-exact routing: every rank computes the same ids), runs its local experts for the
        pairs routed to them and leaves its fp32 share; combine: the exchange kernel sums the
        shares over NVLink peer memory and rank r keeps rows [r*T, (r+1)*T).  With top-8 of 64
        experts over 8 ranks a token reaches ~5.4 of the 8 ranks on average, so gathering every
        row moves ~1.5x the bytes of an exact all-to-all, and needs no per-call exchange of
        counts."""
        T, H = x.shape
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        key = ("gather", T)
        buf = self._gather.get(key)
        if buf is None:
            buf = torch.empty((world * T, H), dtype=x.dtype, device=x.device)
            self._gather[key] = buf
        dist.all_gather_into_tensor(buf, x.contiguous(), group=self.group)
        return self.forward(buf)[rank * T:(rank + 1) * T]

    def close(self):
        for c in self._comms.values():
            c.close()
        self._comms.clear()
        self._gather.clear()
