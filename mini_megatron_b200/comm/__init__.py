"""Communication primitives: autograd collectives, SP collectives, P2P, overlap, symmetric memory."""
from .mappings import (AllReduce, all_reduce, copy_to_model_parallel_region,  # noqa: F401
                       gather_from_model_parallel_region, reduce_from_model_parallel_region,
                       scatter_to_model_parallel_region)
