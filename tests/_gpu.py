"""GPU-side test helpers: numpy <-> device, CUDA graph capture via cuda-python."""
from __future__ import annotations

import numpy as np


def dev(a, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    return t.detach().cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


class Graph:
    """Capture a sequence of launches on a private stream; replay; expose handles."""

    def __init__(self):
        import torch
        from cuda.bindings import runtime as rt
        self.rt = rt
        self.stream = torch.cuda.Stream()
        self.graph = None
        self.exec = None

    def _ok(self, res):
        err = res[0] if isinstance(res, tuple) else res
        assert int(err) == 0, f"cuda runtime error {err}"
        return res[1] if isinstance(res, tuple) and len(res) > 1 else None

    def __enter__(self):
        import torch
        torch.cuda.synchronize()
        self._ok(self.rt.cudaStreamBeginCapture(self.stream.cuda_stream,
                                                self.rt.cudaStreamCaptureMode.cudaStreamCaptureModeThreadLocal))
        return self

    def __exit__(self, exc_type, exc, tb):
        g = self._ok(self.rt.cudaStreamEndCapture(self.stream.cuda_stream))
        self.graph = g
        if exc_type is None:
            self.exec = self._ok(self.rt.cudaGraphInstantiate(g, 0))
        return False

    def last_node(self) -> int:
        """The capture's current single dependency (include/gpu_utils.hpp:45-58)."""
        res = self.rt.cudaStreamGetCaptureInfo(self.stream.cuda_stream)
        assert int(res[0]) == 0, res[0]
        deps = res[4]
        assert len(deps) == 1, deps
        return int(deps[0])

    def launch(self):
        import torch
        self._ok(self.rt.cudaGraphLaunch(self.exec, self.stream.cuda_stream))
        self._ok(self.rt.cudaStreamSynchronize(self.stream.cuda_stream))
        torch.cuda.synchronize()

    @property
    def exec_handle(self) -> int:
        return int(self.exec)

    def close(self):
        if self.exec is not None:
            self.rt.cudaGraphExecDestroy(self.exec)
            self.exec = None
        if self.graph is not None:
            self.rt.cudaGraphDestroy(self.graph)
            self.graph = None
