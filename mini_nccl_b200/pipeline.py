"""Import path kept from mini_nccl (``mini_nccl.pipeline``): this name *is*
:mod:`mini_nccl_b200.parallel.pipeline`, so monkeypatching either affects both."""

import sys

from .parallel import pipeline as _impl

sys.modules[__name__] = _impl
