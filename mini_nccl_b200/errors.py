"""Exception hierarchy.

Same four classes and bases as the reference (mini_nccl/errors.py:11-28), so
``except TimeoutError`` / ``except ConnectionError`` in user code keeps
working.  Native status codes map onto them: a TCP op without progress and a
device-side wait that ran past its ``%globaltimer`` deadline both become
:class:`CollectiveTimeoutError`.
"""

from __future__ import annotations


class MiniNcclError(Exception):
    """Root of every error this library raises on purpose."""


class CollectiveTimeoutError(MiniNcclError, TimeoutError):
    """A peer did not hold up its end of a collective within the op timeout.

    Raised instead of hanging, with the local flight-recorder context in the
    message so the stuck rank and sequence number can be identified.
    """


class PeerClosedError(MiniNcclError, ConnectionError):
    """A peer's connection went away in the middle of a message."""


class RendezvousError(MiniNcclError, TimeoutError):
    """The ranks could not form the full connection mesh."""


class DeviceCommError(MiniNcclError, RuntimeError):
    """A device collective kernel reported a non-timeout error status."""
