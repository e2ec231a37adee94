"""Host-buffer SpMM steps: features in and results out of pinned host memory.

The reference hands the SpMM device buffers only (launchSWTCFSpMM,
src/swtcf_spmm.cu:437-466; spmm_cnic's forward_tensorcore,
TAC_training_backend/spmm_cnic/src/bindings/module.cu:192-197); a caller whose
features live in host memory copies them in and the result out around each
call, one after the other.  ``HostPipeline`` runs such steps -- a forward pass
over X and a second pass over G (the transposed pass of a backward), each with
its host copies -- with the copies overlapped:

* host -> device copies on one stream, device -> host copies on another (the
  host link is full duplex), the passes on a third;
* within a step, G uploads while the forward pass runs and Y downloads while
  the second pass runs;
* across steps, two device buffer sets alternate, so step i + 1's uploads run
  while step i's passes and downloads finish.

``submit`` only enqueues; ``synchronize`` waits for every submitted step.  The
host buffers must be pinned (page-locked) and stay untouched until the step's
copies are done (``synchronize``).
"""
from __future__ import annotations

import torch


class HostPipeline:
    """fwd(X_dev, Y_dev) and bwd(G_dev, Z_dev) enqueue the two passes on the
    current stream (device buffers of shapes x_shape, g_shape, y_shape,
    z_shape, fp32)."""

    def __init__(self, fwd, bwd, x_shape, g_shape, y_shape, z_shape, device=None):
        self.fwd, self.bwd = fwd, bwd
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.device = device
        mk = lambda shape: torch.empty(shape, dtype=torch.float32, device=device)  # noqa: E731
        self.sets = [dict(X=mk(x_shape), G=mk(g_shape), Y=mk(y_shape), Z=mk(z_shape))
                     for _ in range(2)]
        self.h2d = torch.cuda.Stream(device=device)
        self.d2h = torch.cuda.Stream(device=device)
        self.comp = torch.cuda.Stream(device=device)
        ev = lambda: torch.cuda.Event()  # noqa: E731
        for s in self.sets:
            s.update(x_in=ev(), g_in=ev(), y_out=ev(), z_out=ev(), inputs_free=None,
                     outputs_free=None)
        self.i = 0
        self.h2d_bytes = self.d2h_bytes = 0

    def submit(self, hX: torch.Tensor, hG: torch.Tensor, hY: torch.Tensor, hZ: torch.Tensor):
        """Enqueue one step: hX, hG -> device, Y = fwd(X), Z = bwd(G), Y, Z -> hY, hZ."""
        s = self.sets[self.i & 1]
        self.i += 1
        # uploads into this set once the passes of two steps ago stopped reading it
        if s["inputs_free"] is not None:
            self.h2d.wait_event(s["inputs_free"])
        with torch.cuda.stream(self.h2d):
            s["X"].copy_(hX, non_blocking=True)
            s["x_in"].record(self.h2d)
            s["G"].copy_(hG, non_blocking=True)
            s["g_in"].record(self.h2d)
        # passes once the inputs are in and the set's last downloads are done
        self.comp.wait_event(s["x_in"])
        if s["outputs_free"] is not None:
            self.comp.wait_event(s["outputs_free"])
        with torch.cuda.stream(self.comp):
            self.fwd(s["X"], s["Y"])
            s["y_out"].record(self.comp)
            self.comp.wait_event(s["g_in"])
            self.bwd(s["G"], s["Z"])
            s["z_out"].record(self.comp)
            inputs_free = torch.cuda.Event()
            inputs_free.record(self.comp)
        s["inputs_free"] = inputs_free
        # downloads: Y while the second pass runs, then Z
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(s["y_out"])
            hY.copy_(s["Y"], non_blocking=True)
            self.d2h.wait_event(s["z_out"])
            hZ.copy_(s["Z"], non_blocking=True)
            outputs_free = torch.cuda.Event()
            outputs_free.record(self.d2h)
        s["outputs_free"] = outputs_free
        self.h2d_bytes += hX.numel() * hX.element_size() + hG.numel() * hG.element_size()
        self.d2h_bytes += hY.numel() * hY.element_size() + hZ.numel() * hZ.element_size()

    def synchronize(self):
        for st in (self.h2d, self.comp, self.d2h):
            st.synchronize()

    def start_event(self) -> torch.cuda.Event:
        """An event on the upload stream, before the next submitted step."""
        e = torch.cuda.Event(enable_timing=True)
        e.record(self.h2d)
        return e

    def end_event(self) -> torch.cuda.Event:
        """An event after every step submitted so far (all three streams)."""
        self.d2h.wait_stream(self.comp)
        self.d2h.wait_stream(self.h2d)
        e = torch.cuda.Event(enable_timing=True)
        e.record(self.d2h)
        return e
