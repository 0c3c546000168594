"""torchmatch_b200 -- B200-native (sm_100a) batched Jonker-Volgenant.

Importing the package registers the CUDA kernel of
``torch.ops.assignment.jonker_dense_batch`` (a drop-in for the reference
tue-p8n/torchmatch operator of the same name) and exposes the reference's
dispatcher surface under :mod:`torchmatch_b200.assignment`
(``solve``, ``Backend``, ``resolve_backend``, ``ops``).
"""

from __future__ import annotations

from torchmatch_b200 import _loader

_loader.load()

from torchmatch_b200 import assignment  # noqa: E402

__all__ = ["assignment"]
