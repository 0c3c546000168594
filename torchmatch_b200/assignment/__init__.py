"""Linear assignment: the reference's ``torchmatch.assignment`` surface.

``solve`` / ``Backend`` / ``resolve_backend`` route CUDA batches to the
sm_100a ``jonker_dense_batch`` kernel; ``ops`` holds the op handles;
``assignment_cost`` gathers the total cost of a mapping.
"""

from __future__ import annotations

from torchmatch_b200 import _loader

_loader.load()

from torchmatch_b200.assignment import ops  # noqa: E402
from torchmatch_b200.assignment._cost import assignment_cost  # noqa: E402
from torchmatch_b200.assignment._solve import Backend, resolve_backend, solve  # noqa: E402

__all__ = ["Backend", "assignment_cost", "ops", "resolve_backend", "solve"]
