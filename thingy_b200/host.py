"""The fused path over HOST buffers: x in pinned host memory, results back in host memory.

Rows are independent, so the batch is streamed in row chunks through three
CUDA streams: copy-in (H2D) of chunk i+1 and copy-out (D2H) of chunk i-1 run
while the kernel processes chunk i, with two device buffer slots per tensor.
The transfer time over PCIe, not the kernel, bounds this path. Scales for
the whole batch are written into one device buffer (any layout, including
column-major and the swizzled MX layout, whose chunks are then contiguous
slabs or strided columns of it) and copied back once at the end.
"""

from __future__ import annotations

import torch

from .fused import empty_scale
from .layouts import n_groups
from .ops import FP8_DTYPE, launch_rms_norm_fp8


class HostPipeline:
    """Reusable device buffers and streams for :func:`rms_norm_fp8_host`."""

    def __init__(self, H: int, chunk_rows: int, *, residual: bool, device=None):
        self.device = torch.device(device or "cuda")
        self.H = H
        self.chunk = chunk_rows
        dev = self.device
        self.x = [torch.empty(chunk_rows, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.q = [torch.empty(chunk_rows, H, dtype=FP8_DTYPE, device=dev) for _ in range(2)]
        self.res = self.res_out = None
        if residual:
            self.res = [torch.empty_like(self.x[0]) for _ in range(2)]
            self.res_out = [torch.empty_like(self.x[0]) for _ in range(2)]
        self.s_in = torch.cuda.Stream(dev)
        self.s_run = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)
        self._scale_cache: dict = {}

    def device_scale(self, M, group_size, scale_format, scale_layout):
        key = (M, group_size, scale_format, scale_layout)
        if key not in self._scale_cache:
            self._scale_cache[key] = empty_scale(M, self.H, group_size, scale_format,
                                                 scale_layout, self.device)
        return self._scale_cache[key]


def _scale_rows(scale: torch.Tensor, layout: str, r0: int, r1: int, M: int, G: int):
    """The part of a whole-batch scale buffer that holds rows [r0, r1)."""
    if layout == "mx":
        from .layouts import mx_padded_shape

        # r0 is a multiple of 128, so rows [r0, r1) are the swizzled buffer of
        # an (r1 - r0)-row batch starting at byte r0 * padded_columns
        _, cols = mx_padded_shape(M, G)
        return scale[r0 * cols:]
    return scale[r0:r1]


def rms_norm_fp8_host(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    residual: torch.Tensor | None = None,
    out: torch.Tensor,
    scale: torch.Tensor,
    residual_out: torch.Tensor | None = None,
    group_size: int | None = 128,
    scale_format: str = "fp32",
    scale_layout: str = "row",
    pipeline: HostPipeline | None = None,
    chunk_rows: int = 2048,
) -> HostPipeline:
    """Fused [residual add] -> RMSNorm -> FP8 for host tensors (pinned for overlap).

    x, residual, out, residual_out: host [M, H]; scale: host tensor with the
    shape/layout ``empty_scale(M, H, ...)`` returns; weight: device [H].
    Enqueues everything and returns the pipeline (call
    ``torch.cuda.current_stream().synchronize()`` or synchronize the device
    before reading the host outputs); pass the returned pipeline back in to
    reuse its buffers.
    """
    M, H = x.shape
    if scale_layout == "mx" and chunk_rows % 128:
        raise ValueError("chunk_rows must be a multiple of 128 for the swizzled layout")
    if pipeline is None or pipeline.H != H or pipeline.chunk < chunk_rows or (
        (residual is not None) != (pipeline.res is not None)
    ):
        pipeline = HostPipeline(H, chunk_rows, residual=residual is not None,
                                device=weight.device)
    p = pipeline
    chunk = p.chunk
    G = n_groups(H, group_size)
    s_dev = p.device_scale(M, group_size, scale_format, scale_layout)
    main = torch.cuda.current_stream(p.device)
    for s in (p.s_in, p.s_run, p.s_out):
        s.wait_stream(main)
    ev_used = [None, None]   # kernel finished reading slot k
    ev_drained = [None, None]  # copy-out finished reading slot k
    for i, r0 in enumerate(range(0, M, chunk)):
        r1 = min(M, r0 + chunk)
        n = r1 - r0
        k = i % 2
        with torch.cuda.stream(p.s_in):
            if ev_used[k] is not None:
                p.s_in.wait_event(ev_used[k])
            p.x[k][:n].copy_(x[r0:r1], non_blocking=True)
            if residual is not None:
                p.res[k][:n].copy_(residual[r0:r1], non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(p.s_in)
        with torch.cuda.stream(p.s_run):
            p.s_run.wait_event(ev_in)
            if ev_drained[k] is not None:
                p.s_run.wait_event(ev_drained[k])
            launch_rms_norm_fp8(
                p.x[k][:n], weight, eps,
                residual=None if residual is None else p.res[k][:n],
                q=p.q[k][:n],
                scale=_scale_rows(s_dev, scale_layout, r0, r1, M, G),
                residual_out=None if residual_out is None else p.res_out[k][:n],
                group_size=group_size, scale_format=scale_format, scale_layout=scale_layout,
            )  # on p.s_run, the current stream inside this block
            ev_used[k] = torch.cuda.Event()
            ev_used[k].record(p.s_run)
        with torch.cuda.stream(p.s_out):
            p.s_out.wait_event(ev_used[k])
            out[r0:r1].copy_(p.q[k][:n], non_blocking=True)
            if residual_out is not None:
                residual_out[r0:r1].copy_(p.res_out[k][:n], non_blocking=True)
            ev_drained[k] = torch.cuda.Event()
            ev_drained[k].record(p.s_out)
    with torch.cuda.stream(p.s_out):
        p.s_out.wait_stream(p.s_run)
        if scale_layout in ("col", "packed"):  # strided [M, G] / [M, W] views
            scale.copy_(s_dev, non_blocking=True)
        else:
            scale.view(-1).copy_(s_dev.reshape(-1), non_blocking=True)
    main.wait_stream(p.s_out)
    return p
