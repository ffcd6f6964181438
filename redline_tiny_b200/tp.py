"""Peer-memory reductions for the tensor-parallel DiT. PeerRS (W ranks, the default): a reduce-scatter done by the
projection GEMM's own stores, a row-sharded LayerNorm and an all-gather done by that LayerNorm's stores (its
docstring below). PeerReduce (2 ranks): the all-reduce of the out- and down-projection partials fused into the
projection GEMM (which stores its partial into the other rank's memory as it computes it) and the residual +
LayerNorm kernel (which adds the two partials: rl_ln_mod_tp), described here.

The tensor-parallel DiT (the reference itself runs on one device) sums the row-split projections' partial outputs
across ranks before each residual + LayerNorm (one reduction per sublayer, two per block). Here each rank's projection GEMM writes its bf16
partial tile by tile both into its own buffer and, over NVLink, into the other rank's (rl_linear_bfp16_partial: the
partial in 16 x 32 chunks of 1 KB, each sent as one bulk copy; the buffers are cudaMalloc allocations shared by CUDA
IPC handle, plain peer stores), so the transfer overlaps the GEMM's math. A one-thread kernel then stores an epoch number into the other rank's signal pad; the LayerNorm kernel waits
for the other rank's epoch (a bounded wait) and reads both partials from local memory. Each rank sends its partial
once - the bytes a ring all-reduce moves - and no separate collective kernel runs.

The sum is formed in fp32 in rank order and rounded to bf16 before the residual: this equals NCCL's bf16 sum of the
two partials bit for bit.

Buffer layout (per rank, one allocation): [slot 0: partial of rank 0 | of rank 1 | slot 1: same | pads: 2 slots x W
uint64], partials ceil(M / 16) * 16 x D bf16 in the chunk layout. The out- and down-projections alternate between the slots; epochs increase by one per
use. A rank stores into a slot again only after its wait on the other slot has passed, which the other rank signals
after its LayerNorm finished reading the slot. Epochs are kernel arguments, so a CUDA graph of a step would replay
stale epochs: this path is for eager launches only.
"""

import ctypes

import torch

from . import _lib as L

_ALIGN = 256


class PeerReduce:
    """The peer buffers of one tensor-parallel group: this rank's allocation and its mappings of the others'."""

    def __init__(self, group, rank, world, M, D, device):
        import torch.distributed as dist
        if world != 2:
            raise ValueError(f"the peer reduction is built for 2 ranks, not {world}")
        self.rank, self.world, self.M, self.D = rank, world, M, D
        self.part_bytes = ((M + 15) // 16 * 16 * D * 2 + _ALIGN - 1) // _ALIGN * _ALIGN   # whole 16-row chunks
        self.slot_bytes = world * self.part_bytes
        self.pad_off = 2 * self.slot_bytes
        total = self.pad_off + (2 * world * 8 + _ALIGN - 1) // _ALIGN * _ALIGN
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        L.call("rl_ipc_alloc", total, ctypes.byref(ptr), handle)
        self.base = ptr.value
        self.opened = []
        try:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for w, h in enumerate(handles):
                if w == rank:
                    bases.append(self.base)
                    continue
                p = ctypes.c_void_p()
                L.call("rl_ipc_open", (ctypes.c_char * 64).from_buffer_copy(h), ctypes.byref(p))
                self.opened.append(p.value)
                bases.append(p.value)
        except Exception:
            self.close()
            raise
        i64 = dict(dtype=torch.int64, device=device)
        self.peer_base = bases[1 - rank]
        self.parts = [torch.tensor([self.base + s * self.slot_bytes + w * self.part_bytes for w in range(world)], **i64)
                      for s in range(2)]
        self.pads = torch.tensor([b + self.pad_off for b in bases], **i64)
        self.epoch = 0
        self.group = group
        dist.barrier(group=group)       # every rank's pads are zero and mapped before the first signal

    def part(self, slot):
        """(this rank's partial of `slot` here, its copy in the other rank's buffer): where the projection GEMM
        stores its output."""
        off = slot * self.slot_bytes + self.rank * self.part_bytes
        return self.base + off, self.peer_base + off

    def next(self):
        """The (slot, epoch) of the next reduction."""
        self.epoch += 1
        return self.epoch & 1, self.epoch

    def signal(self, slot, epoch, stream):
        L.call("rl_tp_signal", self.pads.data_ptr(), self.world, self.rank, slot, epoch, stream)

    def ln_mod(self, x, slot, epoch, params, row_split, x_out, y, stream):
        """x_out = x + g * bf16(sum of the W partials of `slot`); y = LN(x_out) * scale as bfp16 values (bf16)."""
        pad = self.base + self.pad_off + slot * self.world * 8
        L.call("rl_ln_mod_tp", x.data_ptr(), self.parts[slot].data_ptr(), self.world, pad, self.rank, epoch,
               params.data_ptr(), self.M, self.D, row_split, x_out.data_ptr(), y.data_ptr(), None, stream)

    def close(self):
        """Unmap the peers' buffers and free this rank's; call after a barrier that follows the last use."""
        for p in self.opened:
            L.call("rl_ipc_close", p)
        self.opened = []
        if self.base:
            L.call("rl_ipc_free", self.base)
            self.base = 0


class _DeviceArray:
    """A uint16 (rows, cols) view of memory this module owns (an IPC allocation), through the CUDA array interface
    (no copy)."""

    def __init__(self, ptr, rows, cols):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3, "strides": None}


def peer_rs_layout(M, D, world, rank, bases):
    """The addresses PeerRS hands to the kernels, from every rank's allocation base (`bases`, one int per rank):
    {"bytes": the allocation size, "R": rows per rank, "a_off": offset of the gathered A operand,
    "pad_off": offset of the signal pads, "dsts": [slot][owner] -> where this rank's partial rows for `owner` go
    (in the owner's allocation), "parts": [slot][src] -> this rank's received partial of rank `src`,
    "y_dsts": [owner] -> row R * rank of the owner's A operand, "pads": [owner] -> the owner's pad base}."""
    if M % world or (M // world) % 16:
        raise ValueError(f"peer_rs needs M / world to be a multiple of 16 (M={M}, world={world})")
    R = M // world
    recv_bytes = (R * D * 2 + _ALIGN - 1) // _ALIGN * _ALIGN
    a_off = 2 * world * recv_bytes
    pad_off = a_off + (M * D * 2 + _ALIGN - 1) // _ALIGN * _ALIGN
    total = pad_off + (3 * world * 8 + _ALIGN - 1) // _ALIGN * _ALIGN

    def recv(b, s, src):
        return b + (s * world + src) * recv_bytes

    return {"bytes": total, "R": R, "recv_bytes": recv_bytes, "a_off": a_off, "pad_off": pad_off,
            "dsts": [[recv(bases[o], s, rank) for o in range(world)] for s in range(2)],
            "parts": [[recv(bases[rank], s, w) for w in range(world)] for s in range(2)],
            "y_dsts": [b + a_off + rank * R * D * 2 for b in bases],
            "pads": [b + pad_off for b in bases]}


class PeerRS:
    """Reduce-scatter + row-sharded LayerNorm + all-gather over peer memory for W ranks (reduce_dtype "peer_rs").

    Rank r owns rows [r R, r R + R) of the residual stream (R = M / W, R % 16 == 0). Per sublayer:
    the projection GEMM (rl_linear_bfp16_scatter) stores each 16-row chunk of its bf16 partial, as one 1 KB bulk copy,
    straight into the owning rank's receive buffer (slot s, source r) - every value crosses NVLink once, to its owner,
    while the GEMM computes; rl_tp_signal stores the epoch into every rank's pad [s][r]; rl_ln_mod_tp_rs waits for
    the other ranks' epochs, adds the W partials of its R rows in rank order, applies the residual + LayerNorm and
    stores its rows of y into every rank's copy of the next GEMM's A operand (`a`); rl_tp_signal on slot 2 announces
    them and rl_tp_wait holds the stream until every rank's rows have arrived. Only 1 / W of the LayerNorm runs on a
    rank, and no collective kernel runs.

    Buffer layout (per rank, one allocation): [receive: 2 slots x W sources x R rows x D bf16 (chunk layout) | a: M x
    D bf16 | pads: 3 slots x W uint64]. Ordering: a rank writes into another rank's receive slot s or its `a` only
    after a wait that the other rank's later signal satisfied, and that rank signals only after the kernels that read
    those buffers (stream order), so no write overtakes a read. Epochs are kernel arguments: eager launches only."""

    def __init__(self, group, rank, world, M, D, device):
        import torch.distributed as dist
        lay = peer_rs_layout(M, D, world, rank, [0] * world)       # sizes first: nothing allocated if they fail
        self.rank, self.world, self.M, self.D = rank, world, M, D
        self.R = lay["R"]
        self.r0 = rank * self.R
        self.a_off, self.pad_off = lay["a_off"], lay["pad_off"]
        total = lay["bytes"]
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        L.call("rl_ipc_alloc", total, ctypes.byref(ptr), handle)
        self.base = ptr.value
        self.opened = []
        try:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for w, h in enumerate(handles):
                if w == rank:
                    bases.append(self.base)
                    continue
                p = ctypes.c_void_p()
                L.call("rl_ipc_open", (ctypes.c_char * 64).from_buffer_copy(h), ctypes.byref(p))
                self.opened.append(p.value)
                bases.append(p.value)
        except Exception:
            self.close()
            raise
        i64 = dict(dtype=torch.int64, device=device)
        lay = peer_rs_layout(M, D, world, rank, bases)
        # slot s: where this rank's partial rows for owner o go, and this rank's W received partials
        self.dsts = [torch.tensor(lay["dsts"][s], **i64) for s in range(2)]
        self.parts = [torch.tensor(lay["parts"][s], **i64) for s in range(2)]
        self.y_dsts = torch.tensor(lay["y_dsts"], **i64)
        self.pads = torch.tensor(lay["pads"], **i64)
        self.a = torch.as_tensor(_DeviceArray(self.base + self.a_off, M, D), device=device).view(torch.bfloat16)
        self.epoch = 0
        self.group = group
        dist.barrier(group=group)       # every rank's pads are zero and mapped before the first signal

    def next(self):
        """The (slot, epoch) of the next reduction."""
        self.epoch += 1
        return self.epoch & 1, self.epoch

    def gemm(self, x, w, slot, stream):
        """The projection x @ w (x: M rows), its partial rows sent to their owners' receive slot `slot`."""
        M, K = x.shape
        L.call("rl_linear_bfp16_scatter", x.data_ptr(), M, K, w.native.data_ptr(), w.N, self.dsts[slot].data_ptr(),
               self.world, self.R, stream)

    def signal(self, slot, epoch, stream):
        L.call("rl_tp_signal", self.pads.data_ptr(), self.world, self.rank, slot, epoch, stream)

    def ln_mod(self, x, slot, epoch, params, row_split, x_out, stream):
        """Rows of this rank: x_out = x + g * bf16(sum of the W partials); LN(x_out) * scale into every rank's `a`,
        then the all-gather's signal and wait."""
        pad = self.base + self.pad_off + slot * self.world * 8
        L.call("rl_ln_mod_tp_rs", x.data_ptr(), self.parts[slot].data_ptr(), self.world, pad, self.rank, epoch,
               params.data_ptr(), self.R, self.D, row_split, x_out.data_ptr(), self.y_dsts.data_ptr(), stream)
        self.signal(2, epoch, stream)
        L.call("rl_tp_wait", self.base + self.pad_off + 2 * self.world * 8, self.world, self.rank, epoch, stream)

    def close(self):
        """Unmap the peers' buffers and free this rank's; call after a barrier that follows the last use."""
        self.a = None
        for p in self.opened:
            L.call("rl_ipc_close", p)
        self.opened = []
        if self.base:
            L.call("rl_ipc_free", self.base)
            self.base = 0
