"""Host <-> device step pipeline for serving-style loops.

Every step copies its inputs from pinned host memory to the device, runs the
step on the compute stream and copies its result back to pinned host memory.
:class:`HostDevicePipeline` keeps `depth` device slots and three streams so
that the H2D copy of step i+1 and the D2H copy of step i-1 overlap the compute
of step i; CUDA events order the slots, so the host never synchronises inside
the loop.  Per step and slot:

    h2d stream     : wait compute_done[slot] (step i-depth finished reading it)
                     copy inputs -> slot;            record h2d_done[slot]
    compute stream : wait h2d_done[slot], d2h_done[slot] (output slot drained)
                     out[slot] = fn(*in[slot], out=out[slot]); record compute_done[slot]
    d2h stream     : wait compute_done[slot]
                     copy out[slot] -> host;         record d2h_done[slot]

``run`` brackets the whole loop with CUDA events on the compute stream (the
copy streams start after the start event and the end event waits for the last
D2H), so the elapsed time covers every step's copies.
"""
import torch


class HostDevicePipeline:
    """End-to-end step loop: every step copies its inputs from pinned host
    memory to the device, runs the step, and copies the result back, with `depth`
    device slots and separate host-to-device and device-to-host streams so the
    copies of neighbouring steps overlap the compute."""
    def __init__(self, fn, inputs, output, depth=2, device=None):
        """fn(*device_inputs, out=device_output) runs one step on the current
        stream.  `inputs`: list of (shape, dtype) of the device inputs;
        `output`: (shape, dtype) of the device result."""
        self.fn = fn
        self.depth = depth
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.dev_in = [[torch.empty(s, dtype=d, device=dev) for s, d in inputs] for _ in range(depth)]
        self.dev_out = [torch.empty(output[0], dtype=output[1], device=dev) for _ in range(depth)]
        self.h2d = torch.cuda.Stream(device=dev)
        self.d2h = torch.cuda.Stream(device=dev)
        self.h2d_done = [torch.cuda.Event() for _ in range(depth)]
        self.compute_done = [torch.cuda.Event() for _ in range(depth)]
        self.d2h_done = [torch.cuda.Event() for _ in range(depth)]

    def run(self, steps, host_inputs, host_output, timed=True):
        """Runs `steps` steps; host_inputs(i) -> pinned host tensors of step i,
        host_output(i) -> pinned host tensor that receives step i's result.
        Returns the elapsed device milliseconds (None if not timed)."""
        compute = torch.cuda.current_stream()
        start = torch.cuda.Event(enable_timing=timed)
        end = torch.cuda.Event(enable_timing=timed)
        start.record(compute)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        for i in range(steps):
            b = i % self.depth
            with torch.cuda.stream(self.h2d):
                if i >= self.depth:
                    self.h2d.wait_event(self.compute_done[b])
                for dst, src in zip(self.dev_in[b], host_inputs(i)):
                    dst.copy_(src, non_blocking=True)
                self.h2d_done[b].record(self.h2d)
            compute.wait_event(self.h2d_done[b])
            if i >= self.depth:
                compute.wait_event(self.d2h_done[b])
            self.fn(*self.dev_in[b], out=self.dev_out[b])
            self.compute_done[b].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.compute_done[b])
                host_output(i).copy_(self.dev_out[b], non_blocking=True)
                self.d2h_done[b].record(self.d2h)
        compute.wait_stream(self.d2h)
        compute.wait_stream(self.h2d)
        end.record(compute)
        if not timed:
            return None
        end.synchronize()
        return start.elapsed_time(end)


__all__ = ["HostDevicePipeline"]
