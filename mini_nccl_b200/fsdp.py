"""Import path kept from mini_nccl (``mini_nccl.fsdp``): this name *is*
:mod:`mini_nccl_b200.parallel.fsdp`, so monkeypatching either affects both."""

import sys

from .parallel import fsdp as _impl

sys.modules[__name__] = _impl
