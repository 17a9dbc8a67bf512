"""A minimal FlagGems stand-in over torch.cuda, for running the reference suite on B200.

The reference suite (huangyiqun/triton_chip_benchmarks) reaches the device
only through FlagGems (common.py:20-53, 160-292, 335-534): the vendor name,
the torch device type, the device module that supplies events, graphs and
properties, a device detector with ``support_fp64`` and ``device_count``, and
the backend whose ``matmul`` precision setting it toggles.  FlagGems itself is
not installed in this image; on an NVIDIA GPU each of those is exactly what
torch.cuda provides, so this module maps them one to one and adds nothing.
The reference's own Triton kernels, validation, audits and timing run
unchanged on top of it.
"""

from types import SimpleNamespace

import torch

vendor_name = "nvidia"
device = "cuda"


class _Detector:
    """The device detector the reference queries (common.py:52-53, 217-223)."""

    support_fp64 = True

    @property
    def device_count(self) -> int:
        return torch.cuda.device_count()


runtime = SimpleNamespace(
    torch_device_fn=torch.cuda,
    device=_Detector(),
    torch_backend_device=torch.backends.cuda,
    backend=None,
)
