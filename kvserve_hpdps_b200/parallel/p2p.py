"""Peer-memory primitives of the NVLink data path.

A consumer allocates a receive region with :class:`DeviceRegion` (raw
``cudaMalloc`` memory, so that its CUDA IPC handle covers exactly the
region) and publishes :meth:`DeviceRegion.ipc_handle`.  The producer opens
it with :func:`open_peer` and its kernels store directly into it over
NVLink (``st.global`` to the peer address), then publish a ready flag with a
system-scope release store.  The consumer's kernels wait on the flag with a
bounded spin (``kernels.wait_flag``) before reading.

No TMA multicast and no library kernel ever reads peer memory here: peer
addresses are only written by this framework's own store loops.
"""

from __future__ import annotations

import ctypes

import torch

from kvserve_hpdps_b200.ops._lib import check, lib

IPC_HANDLE_BYTES = 64


class DeviceRegion:
    """Raw device allocation (not owned by PyTorch's caching allocator)."""

    def __init__(self, device: int, nbytes: int, zero: bool = True):
        self.device = int(device)
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        check(lib().kvs_malloc(self.device, self.nbytes, ctypes.byref(p)), "kvs_malloc")
        self.ptr = int(p.value)
        if zero:
            with torch.cuda.device(self.device):
                check(lib().kvs_memset(self.ptr, 0, self.nbytes,
                                       torch.cuda.current_stream().cuda_stream), "memset")
                torch.cuda.current_stream().synchronize()

    def ipc_handle(self) -> bytes:
        buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        n = lib().kvs_ipc_get_handle(self.device, self.ptr, buf)
        if n <= 0:
            raise RuntimeError(f"cudaIpcGetMemHandle failed ({n})")
        return bytes(buf[:n])

    def close(self) -> None:
        if self.ptr:
            lib().kvs_free(self.device, self.ptr)
            self.ptr = 0

    def __del__(self):  # best effort; explicit close() is preferred
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


class PeerMapping:
    """A peer's region opened through its IPC handle (device pointer valid
    on ``device``)."""

    def __init__(self, device: int, handle: bytes, nbytes: int):
        self.device = int(device)
        self.nbytes = int(nbytes)
        buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(handle.ljust(IPC_HANDLE_BYTES, b"\0"))
        p = ctypes.c_void_p()
        check(lib().kvs_ipc_open_handle(self.device, buf, ctypes.byref(p)), "cudaIpcOpenMemHandle")
        self.ptr = int(p.value)

    def close(self) -> None:
        if self.ptr:
            lib().kvs_ipc_close_handle(self.device, self.ptr)
            self.ptr = 0


def open_peer(device: int, handle: bytes, nbytes: int) -> PeerMapping:
    return PeerMapping(device, handle, nbytes)


def can_access_peer(device: int, peer: int) -> bool:
    return lib().kvs_can_access_peer(int(device), int(peer)) == 1


def enable_peer_access(device: int, peer: int) -> None:
    check(lib().kvs_enable_peer_access(int(device), int(peer)), "cudaDeviceEnablePeerAccess")


def read_u32(ptr: int, device: int, count: int = 1) -> list[int]:
    """Host read of ``count`` 32-bit words at a 16-byte aligned device address
    (synchronising)."""
    from kvserve_hpdps_b200.ops import kernels as K
    n16 = (4 * count + 15) // 16
    t = torch.empty(4 * n16, dtype=torch.int32, device=f"cuda:{device}")
    K.copy_bytes(ptr, t.data_ptr(), 16 * n16, torch.device("cuda", device))
    torch.cuda.synchronize(device)
    return [int(x) for x in t[:count].cpu().tolist()]
