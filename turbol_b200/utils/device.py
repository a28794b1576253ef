"""Device-string helpers shared by the Python API."""
from __future__ import annotations

import torch


def parse_device(device) -> torch.device:
    """Accepts torch.device, "cpu", "cuda", "cuda:N", "CPU", "CUDA:N"."""
    if isinstance(device, torch.device):
        return device
    s = str(device).strip().lower()
    if s.startswith("cuda"):
        idx = int(s.split(":", 1)[1]) if ":" in s else 0
        return torch.device("cuda", idx)
    return torch.device("cpu")


def device_str(device) -> str:
    d = parse_device(device)
    return f"cuda:{d.index or 0}" if d.type == "cuda" else "cpu"
