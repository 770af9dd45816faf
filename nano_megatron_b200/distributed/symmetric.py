"""Symmetric device memory across the ranks of one (tensor-parallel) group.

Each rank allocates one zeroed device buffer, exports a CUDA IPC handle, and
opens every peer's handle, so all ranks can load and store every rank's buffer
over NVLink (P2P through NVSwitch). Buffer layout (identical on all ranks):

    [ flags: 16 channels x 8 source slots x uint32 | pad to 4 KiB ]
    [ reduce-scatter tile flags: 8 source slots x 16384 tiles x uint32 ]
    [ reduce-scatter staging: 2 parities x TP x rows x cols bf16 ]
    [ all-gather shards:       2 parities x rows x cols bf16      ]
    [ embedding rows:          2 parities x rows x hidden bf16    ]  (optional)
    [ cross-entropy stats:     2 parities x TP x tokens x 3 fp32  ]  (optional)

A channel's epoch counter lives in device memory (one int per channel, local to
the rank) and is advanced by the signal kernel once per collective call on every
rank (all ranks issue the same calls in the same order); no launch carries the
epoch as an argument, so a step's fused collectives can be captured in a CUDA
graph. Parity = epoch & 1 selects the data half, so call k+1 never overwrites
data call k may still be reading (a rank only reaches call k+2 after every peer
has signalled call k+1, which it does after finishing call k). ``emulated`` builds TP workspaces inside one
process on one GPU -- every "peer" buffer is local -- so the fused kernels'
indexing and reductions can be checked without several GPUs; there the calls
of the emulated ranks are issued phase by phase so no kernel ever waits for a
kernel that has not been launched.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

FLAG_BYTES = 4096
MAX_TP = 8
RS_TILE_FLAGS = 16384              # per source rank; must equal kRsTileFlags (gemm_tcgen05.cu)
TILE_FLAG_BYTES = MAX_TP * RS_TILE_FLAGS * 4
CH_RS, CH_AG, CH_AG_BWD, CH_EMB, CH_CE = 0, 1, 2, 3, 4
GATHER_READY_TILES = 4096          # 128-row tiles of a gathered operand (512K rows)


class SymmetricWorkspace:
    def __init__(self, *, rank: int, size: int, ptrs: list[int], owner: torch.Tensor,
                 device: torch.device, rs_bytes: int, ag_bytes: int, opened: list[int],
                 emb_bytes: int = 0, ce_bytes: int = 0) -> None:
        self.rank, self.size = rank, size
        self.ptrs = ptrs              # base address of every rank's buffer, mapped here
        self.owner = owner            # keeps this rank's allocation alive
        self.device = device
        self.rs_bytes, self.ag_bytes = rs_bytes, ag_bytes
        self.emb_bytes, self.ce_bytes = emb_bytes, ce_bytes
        self._opened = opened         # peer mappings to close
        # one process emulating every rank: kernels of the emulated ranks run one after
        # another, so no kernel may wait inside for another rank's kernel (the
        # reduce-scatter then reduces in a second pass instead of in its epilogue)
        self.emulated = False
        self.epochs = torch.zeros(16, dtype=torch.int32, device=device)  # device counters
        # per channel and 128-row tile: epoch at which the gathered rows sit in the local
        # copy (written and read by the AG->GEMM kernel on this GPU only)
        self.gather_ready = torch.zeros(16, GATHER_READY_TILES, dtype=torch.int32,
                                        device=device)
        from nano_megatron_b200.ops._ext import status_word

        self.status = status_word(device)

    # ------------------------------------------------------------------ construction
    @staticmethod
    def total_bytes(rs_bytes: int, ag_bytes: int, emb_bytes: int = 0, ce_bytes: int = 0) -> int:
        return FLAG_BYTES + TILE_FLAG_BYTES + 2 * (rs_bytes + ag_bytes + emb_bytes + ce_bytes)

    @classmethod
    def create(cls, group, *, rs_bytes: int, ag_bytes: int, device: torch.device,
               emb_bytes: int = 0, ce_bytes: int = 0) -> "SymmetricWorkspace":
        """Collective over ``group`` (a ParallelGroup with an NCCL process group)."""
        from nano_megatron_b200.ops._ext import lib

        if group.size > MAX_TP:
            raise ValueError(f"symmetric workspace supports at most {MAX_TP} ranks")
        rs_bytes, ag_bytes = _align(rs_bytes), _align(ag_bytes)
        emb_bytes, ce_bytes = _align(emb_bytes, 4096, 0), _align(ce_bytes, 4096, 0)
        dev = _indexed(device)
        buf, handle = lib().symm_alloc(cls.total_bytes(rs_bytes, ag_bytes, emb_bytes, ce_bytes),
                                       dev.index)
        handles: list = [None] * group.size
        dist.all_gather_object(handles, bytes(handle), group=group.process_group)
        ptrs, opened = [], []
        for r, h in enumerate(handles):
            if r == group.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = lib().symm_open(h, dev.index)
                opened.append(p)
                ptrs.append(p)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group.process_group, device_ids=[dev.index])
        return cls(rank=group.rank, size=group.size, ptrs=ptrs, owner=buf, device=dev,
                   rs_bytes=rs_bytes, ag_bytes=ag_bytes, opened=opened, emb_bytes=emb_bytes,
                   ce_bytes=ce_bytes)

    @classmethod
    def emulated(cls, size: int, *, rs_bytes: int, ag_bytes: int, device: torch.device,
                 emb_bytes: int = 0, ce_bytes: int = 0) -> list["SymmetricWorkspace"]:
        rs_bytes, ag_bytes = _align(rs_bytes), _align(ag_bytes)
        emb_bytes, ce_bytes = _align(emb_bytes, 4096, 0), _align(ce_bytes, 4096, 0)
        dev = _indexed(device)
        bufs = [torch.zeros(cls.total_bytes(rs_bytes, ag_bytes, emb_bytes, ce_bytes),
                            dtype=torch.uint8, device=dev) for _ in range(size)]
        ptrs = [b.data_ptr() for b in bufs]
        out = [cls(rank=r, size=size, ptrs=ptrs, owner=bufs[r], device=dev, rs_bytes=rs_bytes,
                   ag_bytes=ag_bytes, opened=[], emb_bytes=emb_bytes, ce_bytes=ce_bytes)
               for r in range(size)]
        for ws in out:
            ws.emulated = True
        return out

    def close(self) -> None:
        """Unmap every peer buffer (``cudaIpcCloseMemHandle``). Call only after every peer
        has finished the kernels that store into this rank's view of it (a TP barrier)."""
        if not self._opened:
            return
        from nano_megatron_b200.ops._ext import lib

        opened, self._opened = self._opened, []
        for p in opened:
            lib().symm_close(p, self.device.index)
        self.ptrs = [p if r == self.rank else 0 for r, p in enumerate(self.ptrs)]

    def release(self) -> None:
        """Free this rank's own buffer. Call only after every peer has unmapped it."""
        self.close()
        self.owner = None
        self.ptrs = []

    # ------------------------------------------------------------------ addressing
    def epoch_ptr(self, channel: int) -> int:
        """Device address of this rank's epoch counter for ``channel``."""
        return self.epochs.data_ptr() + 4 * channel

    def flags(self, rank: int, channel: int) -> int:
        return self.ptrs[rank] + channel * MAX_TP * 4

    def signal_targets(self, channel: int) -> list[int]:
        return [self.flags(d, channel) + self.rank * 4 for d in range(self.size)]

    def rs_tile_flags(self, rank: int) -> int:
        """Base of ``rank``'s [source rank][tile] flag array of the in-kernel GEMM ->
        reduce-scatter."""
        return self.ptrs[rank] + FLAG_BYTES

    def _data(self, rank: int) -> int:
        return self.ptrs[rank] + FLAG_BYTES + TILE_FLAG_BYTES

    def rs_staging(self, rank: int, parity: int) -> int:
        return self._data(rank) + (parity & 1) * self.rs_bytes

    def ag_shard(self, rank: int, parity: int) -> int:
        return self._data(rank) + 2 * self.rs_bytes + (parity & 1) * self.ag_bytes

    def emb_slot(self, rank: int, parity: int) -> int:
        return self._data(rank) + 2 * (self.rs_bytes + self.ag_bytes) + \
            (parity & 1) * self.emb_bytes

    def ce_slot(self, rank: int, parity: int) -> int:
        return self._data(rank) + 2 * (self.rs_bytes + self.ag_bytes + self.emb_bytes) + \
            (parity & 1) * self.ce_bytes

    def check_emb(self, rows: int, hidden: int) -> None:
        if rows * hidden * 2 > self.emb_bytes:
            raise ValueError(f"embedding slot needs {rows * hidden * 2} bytes; workspace has "
                             f"{self.emb_bytes}")

    def check_ce(self, tokens: int) -> None:
        if self.size * tokens * 12 > self.ce_bytes:
            raise ValueError(f"cross-entropy statistics need {self.size * tokens * 12} bytes; "
                             f"workspace has {self.ce_bytes}")

    def check_ag(self, rows: int, cols: int) -> None:
        need = rows * cols * 2
        if need > self.ag_bytes:
            raise ValueError(f"all-gather shard needs {need} bytes; workspace has "
                             f"{self.ag_bytes}")

    def check_rs(self, rows: int, cols: int) -> None:
        need = self.size * rows * cols * 2
        if need > self.rs_bytes:
            raise ValueError(f"reduce-scatter staging needs {need} bytes; workspace has "
                             f"{self.rs_bytes}")


def _indexed(device) -> torch.device:
    """``device`` with an explicit CUDA index (``cuda`` alone means the current device)."""
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _align(n: int, a: int = 1 << 21, minimum: int | None = None) -> int:
    up = (int(n) + a - 1) // a * a
    return max(a if minimum is None else minimum, up)


class SymmetricHeap:
    """One IPC-exported device allocation per rank of a group, mapped by every peer and cut
    into named regions at identical offsets on every rank (16-byte aligned). Used by the
    data-parallel replica path for the flat gradient / parameter buffers and their flags.

    ``ptr(rank, name)`` is the device address of ``name`` in ``rank``'s allocation as seen
    from this process; ``local(name, dtype)`` is a tensor view of this rank's region. The
    epoch counters (one per flag channel) are local device memory. Teardown is
    ``close()`` (unmap peers; after a barrier) then ``release()`` (free; after another)."""

    def __init__(self, *, rank: int, size: int, ptrs: list[int], owner, device,
                 offsets: dict[str, tuple[int, int]], opened: list[int]) -> None:
        self.rank, self.size = rank, size
        self.ptrs, self.owner, self.device = ptrs, owner, device
        self.offsets = offsets
        self._opened = opened
        self.epochs = torch.zeros(16, dtype=torch.int32, device=device)
        from nano_megatron_b200.ops._ext import status_word

        self.status = status_word(device)

    @staticmethod
    def layout(regions: dict[str, int]) -> tuple[dict[str, tuple[int, int]], int]:
        offsets, cur = {}, 0
        for name, nbytes in regions.items():
            offsets[name] = (cur, int(nbytes))
            cur += -(-int(nbytes) // 256) * 256
        return offsets, max(cur, 256)

    @classmethod
    def create(cls, group, regions: dict[str, int], device) -> "SymmetricHeap":
        """Collective over ``group`` (rank, size, process_group)."""
        from nano_megatron_b200.ops._ext import lib

        if group.size > MAX_TP:
            raise ValueError(f"symmetric heap supports at most {MAX_TP} ranks")
        offsets, total = cls.layout(regions)
        dev = _indexed(device)
        buf, handle = lib().symm_alloc(total, dev.index)
        handles: list = [None] * group.size
        dist.all_gather_object(handles, bytes(handle), group=group.process_group)
        ptrs, opened = [], []
        for r, h in enumerate(handles):
            if r == group.rank:
                ptrs.append(buf.data_ptr())
            else:
                p = lib().symm_open(h, dev.index)
                opened.append(p)
                ptrs.append(p)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group.process_group, device_ids=[dev.index])
        return cls(rank=group.rank, size=group.size, ptrs=ptrs, owner=buf, device=dev,
                   offsets=offsets, opened=opened)

    @classmethod
    def emulated(cls, size: int, regions: dict[str, int], device) -> list["SymmetricHeap"]:
        """``size`` heaps in one process on one GPU (every "peer" is local memory)."""
        offsets, total = cls.layout(regions)
        dev = _indexed(device)
        bufs = [torch.zeros(total, dtype=torch.uint8, device=dev) for _ in range(size)]
        ptrs = [b.data_ptr() for b in bufs]
        return [cls(rank=r, size=size, ptrs=ptrs, owner=bufs[r], device=dev, offsets=offsets,
                    opened=[]) for r in range(size)]

    def ptr(self, rank: int, name: str) -> int:
        return self.ptrs[rank] + self.offsets[name][0]

    def local(self, name: str, dtype: torch.dtype) -> torch.Tensor:
        off, nbytes = self.offsets[name]
        return self.owner[off:off + nbytes].view(dtype)

    def epoch_ptr(self, channel: int) -> int:
        return self.epochs.data_ptr() + 4 * channel

    def flag_slots(self, rank: int, channel: int) -> int:
        """Address of ``rank``'s flag array for ``channel`` (one uint32 per source rank)."""
        return self.ptr(rank, "flags") + channel * MAX_TP * 4

    def signal_targets(self, channel: int) -> list[int]:
        return [self.flag_slots(d, channel) + self.rank * 4 for d in range(self.size)]

    def close(self) -> None:
        if not self._opened:
            return
        from nano_megatron_b200.ops._ext import lib

        opened, self._opened = self._opened, []
        for p in opened:
            lib().symm_close(p, self.device.index)
        self.ptrs = [p if r == self.rank else 0 for r, p in enumerate(self.ptrs)]

    def release(self) -> None:
        self.close()
        self.owner = None
        self.ptrs = []
