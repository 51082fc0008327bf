"""Device communicator (placeholder until the CUDA runtime lands)."""


class DeviceComm:  # pragma: no cover - replaced by the CUDA implementation
    def __init__(self, comm, global_ranks):
        raise NotImplementedError("device communicator not built yet")
