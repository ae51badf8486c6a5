"""Exception types raised by the runtime."""

from __future__ import annotations

_CODES = {
    1: "mbarrier wait exceeded its cycle budget",
    2: "peer flag never arrived (communication timeout)",
    3: "bounds guard tripped",
    4: "bad device-side argument",
}
_KERNELS = {1: "gemm", 2: "attention", 3: "comm", 4: "norm", 5: "mx", 6: "conv"}


class DeviceError(RuntimeError):
    """A kernel recorded an error in the device error word instead of trapping."""

    def __init__(self, code: int, kernel: int, detail=(0, 0)):
        self.code = int(code)
        self.kernel = int(kernel)
        self.detail = tuple(detail)
        super().__init__(
            f"device error {self.code} ({_CODES.get(self.code, 'unknown')}) in kernel "
            f"{_KERNELS.get(self.kernel, self.kernel)} detail={self.detail}"
        )


class CommTimeoutError(DeviceError):
    """A bounded wait on a peer flag ran out (the peer never signalled)."""


class UnsupportedError(RuntimeError):
    """A configuration the engine refuses, with the reason."""
