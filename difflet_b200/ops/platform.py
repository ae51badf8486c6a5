"""Platform target of the op surface (difflet/ops/platform.py): B200 (sm_100a) or the CPU oracle."""

from enum import Enum

import torch


class hardware(Enum):
    CPU = "cpu"
    B200 = "b200"


def get_platform_target():
    return hardware.B200 if torch.cuda.is_available() else hardware.CPU


def is_cuda() -> bool:
    return torch.cuda.is_available()


__all__ = ["get_platform_target", "hardware", "is_cuda"]
