"""Shared helpers for the parity tests (numpy bit patterns <-> CUDA tensors)."""
import numpy as np
import torch


def to_cuda_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def u8_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def assert_rel(a: float, b: float, rel: float = 1e-5, what: str = ""):
    if np.isinf(b) or np.isinf(a):
        assert a == b, f"{what}: {a} vs {b}"
        return
    assert abs(a - b) <= rel * max(abs(b), 1e-30), f"{what}: {a} vs {b} (rel {abs(a - b) / max(abs(b), 1e-30):.3e})"
