"""kiwi_b200.invoke: host callbacks that running CUDA kernels call.

A :class:`Context` owns ``num_endpoints`` device-to-host rings and a registry
of up to 256 callbacks.  Kernels receive ``ctx.device_context_ptr`` (a
``kiwi::invoke::DeviceContext<Q>*``) and call
``ctx->get_device_handle(ep).invoke(cb_id, args...)`` (see
``include/kiwi/invoke/device_context.cuh``); the host runs the callbacks from
:meth:`Context.progress` or from native progress threads (:meth:`Context.start`).

Python callbacks declare their argument layout with a ``struct`` format
string (little-endian, packed: the layout ``ArgPack`` serialises on the
device), e.g. ``ctx.register_callback(fn, "<Qi")`` for ``invoke(cb, uint64, int32)``.
"""
import struct

from ._native import load as _load

_C = _load()

MAX_CALLBACKS = _C.invoke.MAX_CALLBACKS


class Context:
    """Python face of ``kiwi::invoke::Context<SPSCD2HQueue | MPSCD2HQueue>``."""

    def __init__(self, num_endpoints=1, capacity=4096, mpsc=False, host_only=False):
        self._ctx = _C.invoke.Context(num_endpoints, capacity, mpsc, host_only)
        self.mpsc = mpsc

    # -- registration ------------------------------------------------------
    def register_callback(self, fn, fmt=None):
        """Register ``fn``; returns its 8-bit callback id.

        ``fmt`` None: ``fn(payload: bytes)`` for any payload size.  Otherwise a
        ``struct`` format; the payload must be exactly ``struct.calcsize(fmt)``
        bytes and ``fn`` receives the unpacked values.
        """
        if fmt is None:
            return self._ctx.register_callback(fn, -1)
        if fmt[:1] not in "<=":
            fmt = "<" + fmt  # device serialisation is little-endian and packed
        st = struct.Struct(fmt)

        def thunk(payload, _fn=fn, _st=st):
            _fn(*_st.unpack(payload))

        return self._ctx.register_callback(thunk, st.size)

    def register_native_print(self, fmt, struct_format, stream="stdout"):
        """Register a native (C++, no GIL) callback that prints each invoke's
        arguments: ``struct_format`` gives their packed layout (codes
        b B h H i I l L q Q f d, little-endian) and ``fmt`` a printf-style line
        with one conversion per argument, e.g.
        ``register_native_print("step=%d value=%.2f tag=0x%llx", "<ifQ")``.
        The format is checked against the codes now; returns the callback id."""
        if stream not in ("stdout", "stderr"):
            raise ValueError("stream must be 'stdout' or 'stderr'")
        return self._ctx.register_native_print(fmt, struct_format, stream == "stderr")

    # -- progress ------------------------------------------------------------
    def progress(self, endpoint=0, max_callbacks=-1):
        return self._ctx.progress(endpoint, max_callbacks)

    def progress_all(self, max_per_endpoint=-1):
        return self._ctx.progress_all(max_per_endpoint)

    def start(self, num_threads=1, cpus=None):
        """Start native progress threads pinned to ``cpus`` (default: GPU-local cores)."""
        if cpus is None:
            cpus = []
            if not self._ctx.host_only:
                import torch

                cpus = _C.topology.poller_cpus(torch.cuda.current_device(), num_threads)
        self._ctx.start_progress_threads(num_threads, list(cpus))
        return self

    def stop(self):
        self._ctx.stop_progress_threads()
        self._ctx.rethrow_progress_errors()

    def set_active_endpoints(self, n, wait_s=None):
        """Progress threads poll only endpoints [0, n) (0 = all, the default),
        e.g. the endpoints of the blocks a kernel actually launches.  Growing
        applies at the threads' next sweep; shrinking first drains the dropped
        endpoints once (shrink only after the kernels pushing to them have
        finished).  With ``wait_s``, waits up to that long until every running
        thread has applied the request and raises TimeoutError otherwise.
        Returns the request's generation."""
        import time

        gen = self._ctx.set_active_endpoints(int(n))
        if wait_s is not None:
            deadline = time.monotonic() + wait_s
            while not self._ctx.active_applied(gen):
                if time.monotonic() > deadline:
                    raise TimeoutError("progress threads did not apply the active-endpoint request")
                time.sleep(1e-4)
        return gen

    def register_active_endpoints_callback(self):
        """Registers a native callback taking one uint32 ``n`` that applies
        ``set_active_endpoints(n)``, so a kernel can publish how many endpoints
        it uses with ``invoke(cb, n)``.  Returns the callback id."""
        return self._ctx.register_active_endpoints_callback()

    @property
    def active_endpoints(self):
        """The active prefix requested last (0 = all endpoints)."""
        return self._ctx.active_endpoints

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.stop()
        return False

    # -- introspection ---------------------------------------------------------
    @property
    def device_context_ptr(self):
        """Device address of the ``DeviceContext`` (0 for host-only contexts)."""
        return self._ctx.device_context_ptr

    @property
    def num_endpoints(self):
        return self._ctx.num_endpoints

    @property
    def num_callbacks(self):
        return self._ctx.num_callbacks

    @property
    def callbacks_run(self):
        return self._ctx.callbacks_run

    @property
    def stats(self):
        """Progress-thread totals: ``callbacks``, ``sweeps``, ``empty_polls``
        (endpoint checks that found nothing) and ``threads`` running now."""
        return self._ctx.stats

    @property
    def host_only(self):
        return self._ctx.host_only

    def poll_ready(self, endpoint=0):
        return self._ctx.poll_ready(endpoint)

    def check_device_errors(self):
        self._ctx.check_device_errors()

    def upload_handles(self):
        """Re-upload fresh device handles (every endpoint queue must be drained)."""
        self._ctx.upload_handles()

    def emulate_invoke(self, endpoint, callback_id, payload=b""):
        """Host-only contexts: enqueue a message as a kernel's invoke would."""
        self._ctx.emulate_invoke(endpoint, callback_id, bytes(payload))


__all__ = ["Context", "MAX_CALLBACKS"]
