"""``thin_backend.graph`` (reference thin_backend/graph.py): CapturedForward on CUDA Graphs."""
from thintnpu_b200.graph import CapturedForward, RuntimeGraph  # noqa: F401
