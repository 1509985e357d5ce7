"""panvram_b200 - a B200-native drop-in for panvram's refrel3 v1 random-access window path: a pangenome cohort
resident on the GPU as refrel3 v1 archives (edits against one decoded reference); random windows and coordinate
slices decoded on the card by one sm_100a kernel.

    c = panvram_b200.Cohort.open(dir, device="cuda")  # reference + assemblies resident
    x = c.sample(n, W, generator=g)                    # uint8 [n, W] (bytes or tokens) on the device
    y = c.fetch(assembly, contig, start, length)       # a slice by coordinates
"""
import torch  # noqa: F401  (CUDA context and caching allocator come from torch)

from . import _C
from .cohort import DATASETS, Cohort, global_batch

FormatError = _C.FormatError
with_cuda = _C.with_cuda
__version__ = "0.1.0"
__all__ = ["Cohort", "DATASETS", "FormatError", "with_cuda", "global_batch"]
