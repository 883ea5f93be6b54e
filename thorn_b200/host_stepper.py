"""Optimizer steps fed from, and drained to, pinned host memory.

A training loop that keeps gradients or a parameter mirror in host memory (host-side
gradient accumulation, a parameter server, checkpoint shadows) pays two PCIe
transfers per step.  Run back to back they cost more than the step itself on B200:
an 8B-parameter bf16 model moves 16 GB each way, about 0.3 s per direction at PCIe 5
speeds, against ~0.36 s for the whole THORN step.  ``PinnedStepper`` overlaps them
with the optimizer's own work on two copy streams:

* the gradients of step k are copied host -> device into one of two device gradient
  buffers while step k - 1 still runs;
* after step k the updated parameters are snapshotted device -> device (HBM speed)
  and the snapshot is copied device -> host while step k + 1 runs.

When the host gradient buffers (or the host parameter buffers) are views of one pinned
allocation, in parameter order and of one dtype (:func:`pinned_block` makes them), each
direction is one copy per step instead of one per tensor: hundreds of small copies would
fill the launch queue that the step's kernels also use.  The parameter snapshot is one
multi-tensor device copy either way.

Every dependency is a CUDA event; the host blocks only in :meth:`wait_host_grads` and
:meth:`synchronize`.  Host buffers must be pinned (``torch.empty(..., pin_memory=True)``)
and hold the local shard of every parameter (its ``to_local()`` for a DTensor).  The
host gradients of a step must be written before :meth:`step` is called for it, and not
rewritten until :meth:`wait_host_grads` has returned: the copy that :meth:`step`
enqueues reads them asynchronously.  The host parameter buffers hold the values of
step k once a later :meth:`synchronize` returns.
"""
from __future__ import annotations

import math

import torch

from .optimizer import _local


# Each view of a pinned block starts on this byte boundary, so the device views that mirror
# it start where the kernels' 16-byte vector loads want them.
_ALIGN = 256


def pinned_block(shapes, dtype):
    """One pinned host allocation holding tensors of ``shapes`` in order, each view starting
    on a 256-byte boundary: returns the list of views (pass it to :class:`PinnedStepper` to
    get one copy per direction)."""
    offs, n = _block_layout(shapes, dtype)
    flat = torch.empty(max(1, n), dtype=dtype, pin_memory=True)
    return [flat[o:o + math.prod(s)].view(s) for o, s in zip(offs, shapes)]


def _block_layout(shapes, dtype):
    """Element offsets of the views of :func:`pinned_block` and its length in elements."""
    step = max(1, _ALIGN // torch.empty((), dtype=dtype).element_size())
    offs, n = [], 0
    for s in shapes:
        offs.append(n)
        n += -(-math.prod(s) // step) * step
    return offs, n


def _block_of(ts):
    """``(flat, offsets)``: the span of one storage that holds ``ts`` in order (each
    contiguous, one dtype, ascending and not overlapping; gaps allowed) and the element
    offset of each tensor in it; None when ``ts`` are not laid out that way."""
    if not ts or any(not t.is_contiguous() or t.dtype != ts[0].dtype for t in ts):
        return None
    st = ts[0].untyped_storage()
    if any(t.untyped_storage().data_ptr() != st.data_ptr() for t in ts):
        return None
    base = ts[0].storage_offset()  # in elements: one storage, one dtype
    offs, end = [], base
    for t in ts:
        o = t.storage_offset()
        if o < end:
            return None
        offs.append(o - base)
        end = o + t.numel()
    flat = torch.empty(0, dtype=ts[0].dtype, device=ts[0].device)
    flat.set_(st, base, (end - base,), (1,))
    return flat, offs


class PinnedStepper:
    """Run ``optimizer.step()`` with gradients from ``host_grads`` and the updated
    parameters copied to ``host_params`` (lists in the order of ``params``)."""

    def __init__(self, optimizer, params, host_grads, host_params):
        if not (len(params) == len(host_grads) == len(host_params)):
            raise ValueError("params, host_grads and host_params must have the same length")
        for p, hg, hp in zip(params, host_grads, host_params):
            loc = _local(p)
            if hg.shape != loc.shape or hp.shape != loc.shape:
                raise ValueError(f"host buffers must have the local shape {tuple(loc.shape)}")
            if not (hg.is_pinned() and hp.is_pinned()):
                raise ValueError("host buffers must be pinned (torch.empty(..., pin_memory=True))")
            if hg.dtype != p.dtype or hp.dtype != p.dtype:
                raise TypeError("host buffers must have the parameter dtype")
        self.opt = optimizer
        self.params = list(params)
        self.host_grads = list(host_grads)
        self.host_params = list(host_params)
        dev = _local(self.params[0]).device
        self.device = dev
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        # two gradient buffers (step k fills one while step k - 1 reads the other), one snapshot;
        # when the host buffers form one block, the device buffers mirror its layout
        hg = _block_of(self.host_grads)
        hp = _block_of(self.host_params)
        plain = not any(hasattr(p, "to_local") for p in self.params)  # DTensor grads stay per tensor
        self.h_grads_flat = hg[0] if hg is not None and plain else None
        self.h_params_flat = hp[0] if hp is not None else None
        if self.h_grads_flat is not None:
            self.grads_flat = [torch.empty_like(self.h_grads_flat, device=dev) for _ in range(2)]
            self.grads = [self._views(flat, hg[1]) for flat in self.grads_flat]
        else:
            self.grads_flat = None
            self.grads = [[torch.empty_like(p) for p in self.params] for _ in range(2)]
        if self.h_params_flat is not None:
            self.snapshot_flat = torch.empty_like(self.h_params_flat, device=dev)
            self.snapshot = self._views(self.snapshot_flat, hp[1])
        else:
            self.snapshot_flat = None
            self.snapshot = [torch.empty_like(_local(p)) for p in self.params]
        self.loaded = [torch.cuda.Event(), torch.cuda.Event()]  # gradients of the slot are on the device
        self.consumed = [None, None]  # the step that read the slot has finished
        self.staged = torch.cuda.Event()  # the snapshot holds the latest parameters
        self.drained = None  # the snapshot has been copied to the host
        self.k = 0

    def _views(self, flat, offsets):
        """Views of ``flat`` at ``offsets`` with the local shapes of the parameters."""
        out = []
        for p, off in zip(self.params, offsets):
            shape = _local(p).shape
            out.append(flat[off:off + math.prod(shape)].view(shape))
        return out

    def step(self):
        """Enqueue one step; returns without waiting for the GPU."""
        slot = self.k & 1
        compute = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.h2d):
            if self.consumed[slot] is not None:
                self.h2d.wait_event(self.consumed[slot])
            if self.grads_flat is not None:
                self.grads_flat[slot].copy_(self.h_grads_flat, non_blocking=True)
            else:
                for g, h in zip(self.grads[slot], self.host_grads):
                    _local(g).copy_(h, non_blocking=True)
            self.loaded[slot].record(self.h2d)
        compute.wait_event(self.loaded[slot])
        for p, g in zip(self.params, self.grads[slot]):
            p.grad = g
        self.opt.step()
        done = torch.cuda.Event()
        done.record(compute)
        self.consumed[slot] = done
        if self.drained is not None:
            compute.wait_event(self.drained)  # the host copy of the previous snapshot has finished
        torch._foreach_copy_(self.snapshot, [_local(p).detach() for p in self.params])
        self.staged.record(compute)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self.staged)
            if self.snapshot_flat is not None:
                self.h_params_flat.copy_(self.snapshot_flat, non_blocking=True)
            else:
                for h, s in zip(self.host_params, self.snapshot):
                    h.copy_(s, non_blocking=True)
            drained = torch.cuda.Event()
            drained.record(self.d2h)
        self.drained = drained
        self.k += 1

    def wait_host_grads(self):
        """Block until the host gradients handed to the last :meth:`step` have been
        copied to the device, so the caller may write the next step's gradients.  The
        GPU keeps computing meanwhile."""
        if self.k:
            self.loaded[(self.k - 1) & 1].synchronize()

    def wait_on(self, stream=None):
        """Make ``stream`` (default: the current one) wait until every enqueued
        transfer and step has finished, without blocking the host."""
        stream = stream or torch.cuda.current_stream(self.device)
        if self.drained is not None:
            stream.wait_event(self.drained)
        for ev in self.consumed:
            if ev is not None:
                stream.wait_event(ev)

    def synchronize(self):
        """Block until the host parameter buffers hold the latest step's values."""
        self.wait_on()
        torch.cuda.current_stream(self.device).synchronize()
