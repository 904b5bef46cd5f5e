"""The pyopencl subset that the reference's trainer and CLI call directly, over CUDA streams and
events -- so that MolSzabi/ffnerf-experimental's own ``run_ffnerf_OG.py`` and ``ffnerf_cli.py``
run unmodified on libffnerf.so (together with this package's ``ffnerf_tools`` and the headless
``render_nerf`` beside this module; ``run_reference.py`` puts all three on the import path).

Call sites covered (reference file:line): ``import pyopencl as cl`` (run_ffnerf_OG.py:28);
``cl.Event`` / ``cl.command_execution_status.COMPLETE`` (:696-702, 1304, 1333);
``cl.enqueue_copy`` host->device with ``wait_for`` (:752-753, 1221, 1262, 1454, 1486) and
device->host (:1379); ``cl.wait_for_events`` (:1145, 1153, 1377); ``cl.Context([dev])`` (:1036;
render_nerf.py:373); ``queue.finish()`` (:1512, 1563, the queue comes from ffnerf_tools.make_queue).

Semantics.  A queue is one in-order CUDA stream, so "out-of-order" queues execute in order and
event dependencies are always met.  ``enqueue_copy`` of host memory copies through a private
pinned staging buffer: with the default ``is_blocking=True`` the host array may be reused as soon
as the call returns (pyopencl's contract); a device->host copy waits for its data.  Device buffers
are the torch CUDA tensors that ``ffnerf_tools.RayBatch`` and ``Nerf`` hold; copies are byte-for-
byte (a structured ray array of 32-byte records lands in a [n, 8] float32 buffer unchanged).
"""
from __future__ import annotations

import numpy as np

import ffnerf_tools as _ft

Event = _ft.Event
Context = _ft.Context
CommandQueue = _ft.CommandQueue
Device = _ft.Device
Platform = _ft.Platform


class command_execution_status:          # cl.command_execution_status
    COMPLETE = 0
    RUNNING = 1
    SUBMITTED = 2
    QUEUED = 3


class command_queue_properties:          # cl.command_queue_properties
    OUT_OF_ORDER_EXEC_MODE_ENABLE = 1
    PROFILING_ENABLE = 2


class mem_flags:                         # cl.mem_flags (accepted and ignored: buffers are torch tensors)
    READ_WRITE = 1
    WRITE_ONLY = 2
    READ_ONLY = 4
    USE_HOST_PTR = 8
    ALLOC_HOST_PTR = 16
    COPY_HOST_PTR = 32


def get_platforms():
    return [Platform()]


def create_some_context(interactive=None, answers=None):
    """The first CUDA device (there is no interactive choice)."""
    return Context([_ft.pick_first_device()[1]])


def _is_device(x) -> bool:
    import torch
    return isinstance(x, torch.Tensor) and x.is_cuda


def _bytes_view(t):
    """A flat uint8 view of a contiguous tensor."""
    return t.reshape(-1).view(__import__("torch").uint8)


def enqueue_copy(queue, dest, src, wait_for=None, is_blocking: bool = True, **_kw) -> Event:
    """Copies src into dest on ``queue`` after the events in ``wait_for``; returns the copy's event.
    Host arrays are numpy arrays, device buffers torch CUDA tensors; sizes are in bytes and must match."""
    import torch
    queue.wait_for([e for e in (wait_for or []) if e is not None])
    d_dev, s_dev = _is_device(dest), _is_device(src)
    with torch.cuda.stream(queue.stream):
        if d_dev and s_dev:
            db, sb = _bytes_view(dest), _bytes_view(src)
            if db.numel() != sb.numel():
                raise ValueError(f"enqueue_copy: {sb.numel()} source bytes into {db.numel()} destination bytes")
            db.copy_(sb, non_blocking=True)
            return Event(queue.stream)
        if d_dev:
            host = np.ascontiguousarray(src)
            hb = host.reshape(-1).view(np.uint8)
            db = _bytes_view(dest)
            if hb.size != db.numel():
                raise ValueError(f"enqueue_copy: {hb.size} host bytes into a {db.numel()}-byte device buffer")
            stage = torch.from_numpy(hb.copy()).pin_memory()      # the host array is free on return
            db.copy_(stage, non_blocking=True)
            ev = Event(queue.stream)
            ev._keep = stage                                       # the staging buffer lives with the event
            return ev
        if s_dev:
            out = np.asarray(dest)
            if not out.flags.c_contiguous or not out.flags.writeable:
                raise ValueError("enqueue_copy: the host destination must be a writable contiguous array")
            sb = _bytes_view(src)
            ob = out.reshape(-1).view(np.uint8)
            if ob.size != sb.numel():
                raise ValueError(f"enqueue_copy: {sb.numel()} device bytes into a {ob.size}-byte host array")
            stage = torch.empty(sb.numel(), dtype=torch.uint8, pin_memory=True)
            stage.copy_(sb, non_blocking=True)
            ev = Event(queue.stream)
            ev.wait()                                              # the host array is valid on return
            ob[...] = stage.numpy()
            return ev
    raise TypeError("enqueue_copy: host-to-host copies are not supported")


def wait_for_events(events):
    for e in events or []:
        if e is not None:
            e.wait()
