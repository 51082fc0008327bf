"""Import path kept from mini_nccl (``mini_nccl.tensor_parallel``): this name *is*
:mod:`mini_nccl_b200.parallel.tensor_parallel`, so monkeypatching either affects both."""

import sys

from .parallel import tensor_parallel as _impl

sys.modules[__name__] = _impl
