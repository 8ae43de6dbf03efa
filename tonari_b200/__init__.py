"""tonari_b200 -- B200-native (sm_100a) CUDA provider of tonari's neighbor list."""
from .api import neighbor_list
from .graph import neighbor_graph
from .verlet import VerletNeighborList

__version__ = "0.1.0"
__all__ = ["neighbor_list", "neighbor_graph", "VerletNeighborList"]
