"""Device-buffer helpers for the GPU tests (torch is used only for memory and streams)."""
import numpy as np


def dev(torch, a: np.ndarray):
    """numpy array -> contiguous device tensor with the same bytes."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16).copy())
    elif a.dtype == np.uint32:
        t = torch.from_numpy(a.view(np.int32).copy())
    else:
        t = torch.from_numpy(a.copy())
    return t.cuda()


def host(t, dtype=None) -> np.ndarray:
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def zeros(torch, shape, dtype):
    m = {np.float32: torch.float32, np.uint16: torch.int16, np.uint32: torch.int32, np.float64: torch.float64}
    return torch.zeros(shape, dtype=m[dtype], device="cuda")
