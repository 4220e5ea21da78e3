"""Cross-GPU session migration: move a checkpoint to another GPU by a peer copy over NVLink.

Sessions are independent (the reference serves one session per graph set, README.md:158), so a
multi-GPU deployment spreads sessions over GPUs and keeps each checkpoint on the GPU that made
it (fastworld/prefix_cache.py:85-87 stores ``rt.state()`` in the radix tree).  Restoring a
branch on another GPU needs that checkpoint there: the owner process exports the snapshot's
device buffer through a CUDA IPC handle (exchanged over a host-side process group), the
receiver maps it and pulls the bytes with the engine's vectorised copy kernel, whose loads
read the peer's HBM directly over NVLink (``fw_copy`` with a peer source).  No collective
touches the data path: only the 100-byte handle crosses the host process group.
"""
from __future__ import annotations

from typing import Any, Tuple

import torch

from ._lib import check, lib, ptr, stream_ptr


def export_blob(blob: torch.Tensor) -> Tuple[Any, ...]:
    """IPC description of a device buffer (the storage handle plus this tensor's byte range)."""
    if not blob.is_cuda or not blob.is_contiguous():
        raise ValueError("export_blob: contiguous CUDA tensor required")
    st = blob.untyped_storage()
    meta = st._share_cuda_()
    return (meta, blob.storage_offset() * blob.element_size(), blob.numel() * blob.element_size())


def import_blob(desc: Tuple[Any, ...]) -> torch.Tensor:
    """Map a peer's exported buffer into this process (read-only use); returns a uint8 view."""
    meta, off, nbytes = desc
    st = torch.UntypedStorage._new_shared_cuda(*meta)
    t = torch.empty(0, dtype=torch.uint8, device=st.device)
    t.set_(st, 0, (st.size(),), (1,))
    return t[off:off + nbytes]


def pull(dst: torch.Tensor, src_peer: torch.Tensor) -> torch.Tensor:
    """Copy a peer GPU's buffer into a local one with the engine's copy kernel (runs on the
    destination GPU, reads over NVLink)."""
    nb = dst.numel() * dst.element_size()
    if src_peer.numel() * src_peer.element_size() != nb:
        raise ValueError("pull: byte sizes differ")
    with torch.cuda.device(dst.device):
        check(lib().fw_copy(ptr(dst), ptr(src_peer), nb, stream_ptr()), "fw_copy(peer)")
    return dst


def migrate_state(session, desc) -> None:
    """Restore a session from a snapshot that lives on another GPU (exported with
    :func:`export_blob` of ``SessionState.blob``)."""
    peer = import_blob(desc)
    pull(session._blob, peer)
