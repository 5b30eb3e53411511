"""Helpers shared by the GPU tests (moving oracle inputs to the device)."""

import numpy as np
import torch


def dev(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)


def host(t):
    return t.float().cpu().numpy()


class force_generic:
    """Context manager routing every call to the generic kernels."""

    def __enter__(self):
        from llms_b200 import _capi
        self.prev = _capi.lib.b200mm_force_generic(1)

    def __exit__(self, *exc):
        from llms_b200 import _capi
        _capi.lib.b200mm_force_generic(self.prev)
