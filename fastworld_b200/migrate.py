"""Cross-GPU session migration: move a checkpoint to another GPU by a peer copy over NVLink.

Sessions are independent (the reference serves one session per graph set, README.md:158), so a
multi-GPU deployment spreads sessions over GPUs and keeps each checkpoint on the GPU that made
it (fastworld/prefix_cache.py:85-87 stores ``rt.state()`` in the radix tree).  Restoring a
branch on another GPU needs that checkpoint there: the owner process exports the snapshot's
device allocation as a CUDA IPC handle (exchanged over a host-side process group); the receiver
maps it into its OWN device's address space with peer access enabled (``fw_ipc_open``) and pulls
the bytes with the engine's vectorised copy kernel, whose loads read the owner's HBM over
NVLink.  No collective touches the data path: only the handle crosses the host process group.
"""
from __future__ import annotations

import ctypes
from typing import Any, Dict

import torch

from ._lib import check, lib, ptr, stream_ptr


def export_blob(blob: torch.Tensor) -> Dict[str, Any]:
    """IPC description of a device buffer: the handle of its allocation and the byte range.
    The owner must keep ``blob`` alive until every receiver has finished pulling."""
    if not blob.is_cuda or not blob.is_contiguous():
        raise ValueError("export_blob: contiguous CUDA tensor required")
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_size_t()
    with torch.cuda.device(blob.device):
        check(lib().fw_ipc_get_handle(ptr(blob), buf, ctypes.byref(off)), "fw_ipc_get_handle")
    return {"device": blob.device.index, "handle": buf.raw, "offset": off.value,
            "nbytes": blob.numel() * blob.element_size()}


class PeerBuffer:
    """An exported peer buffer mapped into the current device's address space (context manager)."""

    def __init__(self, desc: Dict[str, Any], device):
        self.desc, self.device, self.base = desc, torch.device(device), ctypes.c_void_p()

    def __enter__(self):
        with torch.cuda.device(self.device):
            check(lib().fw_ipc_open(self.desc["handle"], ctypes.byref(self.base)), "fw_ipc_open")
        return self

    @property
    def ptr(self) -> int:
        return self.base.value + self.desc["offset"]

    def __exit__(self, *exc):
        with torch.cuda.device(self.device):
            torch.cuda.current_stream().synchronize()
            check(lib().fw_ipc_close(self.base), "fw_ipc_close")


def pull(dst: torch.Tensor, peer: PeerBuffer) -> torch.Tensor:
    """Copy a mapped peer buffer into ``dst`` on dst's GPU with the engine's copy kernel (its
    loads read the owner's HBM over NVLink); asynchronous on the current stream."""
    nb = dst.numel() * dst.element_size()
    if nb != peer.desc["nbytes"] or not dst.is_contiguous():
        raise ValueError("pull: byte sizes differ or dst not contiguous")
    with torch.cuda.device(dst.device):
        check(lib().fw_copy(ptr(dst), peer.ptr, nb, stream_ptr()), "fw_copy(peer)")
    return dst


def pull_into(dst: torch.Tensor, desc: Dict[str, Any]) -> torch.Tensor:
    """Map, copy and unmap (synchronises before unmapping)."""
    with PeerBuffer(desc, dst.device) as peer:
        pull(dst, peer)
    return dst


def pull_local(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Same-GPU copy with the engine's copy kernel (checkpoint save / restore)."""
    nb = dst.numel() * dst.element_size()
    check(lib().fw_copy(ptr(dst), ptr(src), nb, stream_ptr()), "fw_copy")
    return dst


def migrate_state(session, desc: Dict[str, Any]) -> None:
    """Restore a session from a snapshot that lives on another GPU (``export_blob`` of a
    ``SessionState.blob``)."""
    pull_into(session._blob, desc)
