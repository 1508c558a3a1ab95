"""``blocked_graph`` (reference blocked_graph.py:4-23): FrozenGraph and its region contract."""
from thintnpu_b200.graph import FrozenGraph, RegionContract  # noqa: F401
