"""Import path kept from mini_nccl (``mini_nccl.ddp``): this name *is*
:mod:`mini_nccl_b200.parallel.ddp`, so monkeypatching either affects both."""

import sys

from .parallel import ddp as _impl

sys.modules[__name__] = _impl
