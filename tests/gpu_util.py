"""Device-buffer helpers for the GPU tests (torch allocates; kernels run through the C ABI)."""
import numpy as np
import torch


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def empty_f32(n: int) -> torch.Tensor:
    return torch.empty(n, dtype=torch.float32, device="cuda")


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()
