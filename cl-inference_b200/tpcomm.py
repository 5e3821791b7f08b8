"""Tensor-parallel groups for the fused GEMV + all-reduce (clq_linear_allreduce_device).

One process per GPU.  Each rank allocates its receive buffer and epoch block
in libclq, exports the buffer as a CUDA IPC handle, and maps every other
rank's; the
handle exchange is any all-gather of Python objects (torch.distributed's
all_gather_object in practice).  The kernel then writes each rank's partial
outputs straight into every rank's buffer over NVLink as 8-byte (epoch, value)
words and sums them, so a row-parallel linear needs no separate collective.
"""
import ctypes

from . import _lib
from .store import _XTYPE, current_stream_handle


class TpComm:
    """RANK of WORLD; EXCHANGE(obj) returns the list of every rank's OBJ in rank order.
    CAP bounds the outputs one SM produces per call (16 x activation rows per
    16-row tile it owns); each rank's buffer is 2 x WORLD x 160 x CAP x 8 bytes."""

    def __init__(self, rank, world, exchange, cap=4096):
        lib = _lib.lib
        self.rank, self.world, self.cap = int(rank), int(world), int(cap)
        recv, flags = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(lib.clq_tp_buffers(self.world, self.cap, ctypes.byref(recv), ctypes.byref(flags)))
        self._local = (recv, flags)
        self._opened = []
        self._handle = None
        try:
            mine = b""
            if self.world > 1:
                hr = (ctypes.c_uint8 * 64)()
                _lib.check(lib.clq_ipc_handle(recv, hr))
                mine = bytes(hr)
            handles = exchange(mine)
            if len(handles) != self.world:
                raise ValueError(f"exchange returned {len(handles)} entries for {self.world} ranks")
            R, F = (ctypes.c_void_p * self.world)(), (ctypes.c_void_p * self.world)()
            for r, hr_b in enumerate(handles):
                F[r] = flags.value  # only this rank's epoch block is read
                if r == self.rank:
                    R[r] = recv.value
                    continue
                pr = ctypes.c_void_p()
                _lib.check(lib.clq_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(hr_b), ctypes.byref(pr)))
                self._opened.append(pr)
                R[r] = pr.value
            h = ctypes.c_void_p()
            _lib.check(lib.clq_tp_create(self.rank, self.world, self.cap, R, F, ctypes.byref(h)))
            self._handle = h
        except BaseException:
            self._release()
            raise

    def linear_allreduce(self, store, x, out=None, row_begin=0, rows=None, stream=None):
        """out[m, rows] = sum over ranks of x_r . W_r[row_begin:row_begin+rows]^T (every rank gets it)."""
        import torch
        if self._handle is None:
            raise ValueError("group is closed")
        rows = store.n - row_begin if rows is None else rows
        if x.dim() != 2 or x.shape[1] != store.k or not x.is_cuda:
            raise ValueError(f"x must be a CUDA [m, {store.k}] matrix, got {tuple(x.shape)}")
        x = x.contiguous()
        m = x.shape[0]
        if out is None:
            out = torch.empty((m, rows), dtype=torch.float32, device=x.device)
        xtype = _XTYPE.get(str(x.dtype).replace("torch.", ""))
        if xtype is None:
            raise ValueError(f"unsupported activation dtype {x.dtype}")
        _lib.check(_lib.lib.clq_linear_allreduce_device(store.handle, row_begin, rows, x.data_ptr(), xtype, m,
                                                        out.data_ptr(), out.stride(0), self._handle,
                                                        stream if stream is not None else current_stream_handle()))
        return out

    def _release(self):
        lib = _lib.lib
        if self._handle is not None:
            lib.clq_tp_free(self._handle)
            self._handle = None
        for ptr in self._opened:
            lib.clq_ipc_close(ptr)
        self._opened = []
        if self._local is not None:
            lib.clq_tp_buffers_free(*self._local)
            self._local = None

    def close(self, barrier=None):
        """Release the group; BARRIER (e.g. dist.barrier) keeps peers from writing into freed memory."""
        if barrier is not None:
            barrier()
        self._release()
