"""Fully sharded data parallelism (ZeRO-3 style).

Semantics of the reference FSDP (mini_nccl/fsdp.py:1-389): every child module
matching ``unit_cls`` (or listed in ``units``) becomes a *unit* whose
parameters are flattened, padded to a multiple of the world size and split so
rank ``r`` keeps shard ``r`` as its only persistent copy.  Forward gathers
the full flat parameters, runs the unit without building a graph and drops
them again; backward gathers again, **recomputes** the unit's forward with the
CPU and CUDA generator states rewound (so dropout replays the same mask),
takes gradients, reduce-scatters them and divides by ``W``.  Parameters
outside any unit stay replicated and are averaged in ``sync()``.  The
optimizer sees shards and replicated parameters only, so parameters,
gradients and optimizer state all scale as ``1/W``.

On CUDA the shards live in the group's symmetric device memory: the gather is
one peer-memory kernel that *pulls* every rank's shard straight into the
destination buffer (no staging copy), and the gradient reduce-scatter reads
peers' gradient buffers directly and applies the ``1/W`` scale in its
epilogue.  ``prefetch=True`` issues the next unit's gather on a side stream
while the current unit computes.

``recompute=False`` keeps the forward's activations instead (torch FSDP2's
default): the gathered parameters are still freed after each unit's forward
-- their storage shrinks to zero bytes -- and gathered back into the same
storage by a hook just before the unit's backward, so saved tensors stay
valid; each unit's gradients are reduce-scattered as soon as all of them
have accumulated.  Peak memory then holds activations rather than extra
compute.

``fuse_gather_gemm=True`` (with ``recompute=False``, on GPUs) gathers each
unit's parameters inside its first GEMM: one kernel whose extra warps copy
the unit's flat buffer in from every rank's shard -- the first GEMM's weight
first -- while its MMAs start on the tiles whose weight rows have arrived
(:meth:`DeviceComm.gather_weight_gemm`).  The unit provides the hook
(``fsdp_first_gemm`` / ``fsdp_forward_with_gathered_gemm``, as the GPT block
does); its 1-D parameters stay whole on every rank so that its LayerNorm can
run before anything is gathered.

``optimizer_in_backward=dict(lr=..., betas=..., eps=..., weight_decay=...)``
fuses the shard's AdamW step into the gradient reduce-scatter: on CUDA one
kernel pushes every gradient chunk to its owner, sums the W slots in rank
order and updates the fp32 master shard and moments in the same pass (the
reduced gradient never touches memory); shards then carry no ``.grad`` and
the user's optimizer only steps the replicated parameters.  The update is the
same decoupled-weight-decay AdamW as ``ops.kernels.FusedAdamW``; ``lr`` may be
changed between steps through :attr:`FullyShardedDataParallel.shard_optimizer`.
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Iterator

import torch
from torch import nn

from .. import collectives
from ..communicator import Communicator
from .ddp import average_gradients

_RELEASED = torch.empty(0)

#: Flatten each unit's gradients into one of two alternating buffers bound to
#: the NVLS multicast object, so the reduce-scatter (and fused AdamW) reads
#: them in place through the switch: no zero fill of a fresh buffer and no
#: copy into a staging buffer.  "0" flattens into ordinary device memory.
FSDP_NVLS_GRADS = os.environ.get("MINI_NCCL_FSDP_NVLS_GRADS", "1") != "0"


class _Unit:
    """One module whose parameters are sharded across ranks."""

    def __init__(self, module: nn.Module, pg: Communicator, name: str, keep_vectors_whole: bool = False) -> None:
        self.module = module
        self.pg = pg
        self.name = name
        self.owner: FullyShardedDataParallel | None = None
        # (owning submodule, attribute, shape, numel); a tied parameter appears once.
        self.entries: list[tuple[nn.Module, str, torch.Size, int]] = []
        self.params: list[nn.Parameter] = []
        seen: set[int] = set()
        for sub in module.modules():
            for attr, p in list(sub.named_parameters(recurse=False)):
                if id(p) in seen or (keep_vectors_whole and p.dim() < 2):
                    continue
                seen.add(id(p))
                self.entries.append((sub, attr, p.shape, p.numel()))
                self.params.append(p)
        dtypes = {p.dtype for p in self.params}
        if len(dtypes) > 1:
            raise ValueError(f"unit {name!r} mixes dtypes {dtypes}; shard them separately")
        self.dtype = self.params[0].dtype if self.params else torch.float32
        self.device = self.params[0].device if self.params else torch.device("cpu")
        W = pg.world_size
        self.total_numel = sum(e[3] for e in self.entries)
        # CUDA shards are a multiple of 8 elements (16-byte vector access in the kernels)
        quantum = W * (8 if self.device.type == "cuda" else 1)
        self.padded_numel = -(-self.total_numel // quantum) * quantum
        self.shard_numel = self.padded_numel // W

        flat = torch.zeros(self.padded_numel, dtype=self.dtype, device=self.device)
        at = 0
        for p, (_, _, _, n) in zip(self.params, self.entries, strict=True):
            flat[at : at + n].copy_(p.detach().reshape(-1))
            at += n
        mine = flat[pg.rank * self.shard_numel : (pg.rank + 1) * self.shard_numel]
        if self.device.type == "cuda" and W > 1:
            store = pg.device_comm().symmetric_zeros(self.shard_numel, self.dtype)
            store.copy_(mine)
            self.shard = nn.Parameter(store)
        else:
            self.shard = nn.Parameter(mine.clone())
        self.release()

    @property
    def full_bytes(self) -> int:
        return self.padded_numel * self.shard.element_size()

    def _gather(self, shard: torch.Tensor) -> torch.Tensor:
        if self.pg.world_size == 1:
            return shard.detach().reshape(-1)
        out = torch.empty(self.padded_numel, dtype=self.dtype, device=shard.device)
        return collectives.all_gather_into(self.pg, out, shard.detach())

    def _bind(self, flat: torch.Tensor) -> None:
        at = 0
        for sub, attr, shape, n in self.entries:
            param = sub._parameters[attr]
            assert param is not None
            param.data = flat[at : at + n].view(shape)
            at += n

    def materialize(self, shard: torch.Tensor, flat: torch.Tensor | None = None) -> torch.Tensor:
        """Gather (unless ``flat`` was prefetched) and point the params at it."""
        if flat is None:
            flat = self._gather(shard)
        self._bind(flat)
        if self.owner is not None:
            self.owner._note_materialized(self.full_bytes)
        return flat

    def release(self) -> None:
        for sub, attr, _, _ in self.entries:
            param = sub._parameters[attr]
            assert param is not None
            param.data = _RELEASED
        if self.owner is not None:
            self.owner._note_released(self.full_bytes)

    def reduce_scatter_grads(self, grads: tuple[torch.Tensor | None, ...]) -> torch.Tensor:
        """Flatten the unit's gradients, keep this rank's averaged slice."""
        W = self.pg.world_size
        flat = self.owner._grad_buffer(self) if self.owner is not None and W > 1 else None
        if flat is not None:  # multicast-bound, reused: zero only what no gradient covers
            at = 0
            for g, (_, _, _, n) in zip(grads, self.entries, strict=True):
                if g is None:
                    flat[at : at + n].zero_()
                else:
                    flat[at : at + n].copy_(g.reshape(-1))
                at += n
            if at < self.padded_numel:
                flat[at:].zero_()
        else:
            if self.device.type == "cuda" and W > 1:
                flat = self.pg.device_comm().scratch_zeros(self.padded_numel, self.dtype)
            else:
                flat = torch.zeros(self.padded_numel, dtype=self.dtype, device=self.device)
            at = 0
            for g, (_, _, _, n) in zip(grads, self.entries, strict=True):
                if g is not None:
                    flat[at : at + n].copy_(g.reshape(-1))
                at += n
        opt = self.owner.shard_optimizer if self.owner is not None else None
        if opt is not None:
            opt.step_unit(self, flat)
            return None
        if W == 1:
            return flat
        if flat.is_cuda:
            return self.pg.device_comm().reduce_scatter(flat, op="sum", scale=1.0 / W)
        return collectives.reduce_scatter(self.pg, flat, op="sum").div_(W)

    def gather_full_flat(self) -> torch.Tensor:
        return self._gather(self.shard)

    # ---- no-recompute mode: activations saved, parameters resharded in between ----

    def _offset_of(self, param: nn.Parameter) -> int:
        at = 0
        for p, (_, _, _, n) in zip(self.params, self.entries, strict=True):
            if p is param:
                return at
            at += n
        raise ValueError("the first GEMM's weight is not one of the unit's sharded parameters")

    def fused_gather_ok(self, x: torch.Tensor) -> bool:
        owner = self.owner
        return (owner is not None and owner.fuse_gather_gemm and x.is_cuda and self.pg.world_size > 1
                and self.dtype == torch.bfloat16 and hasattr(self.module, "fsdp_forward_with_gathered_gemm"))

    def _forward_gathering_in_first_gemm(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Bind the parameters to a fresh buffer that the unit's first GEMM fills."""
        flat = torch.empty(self.padded_numel, dtype=self.dtype, device=self.device)
        self._bind(flat)  # views now; their values arrive inside the first GEMM's kernel
        if self.owner is not None:
            self.owner._note_materialized(self.full_bytes)
        weight, bias = self.module.fsdp_first_gemm()
        w_off = self._offset_of(weight)
        dc = self.pg.device_comm()
        shard = self.shard.detach()

        def gather_gemm(x2: torch.Tensor) -> torch.Tensor:
            return dc.gather_weight_gemm(x2, shard, flat, w_off, weight.shape[0], bias=bias)

        return self.module.fsdp_forward_with_gathered_gemm(x, gather_gemm), flat

    def forward_saving_activations(self, x: torch.Tensor) -> torch.Tensor:
        """Forward with the autograd graph kept; the gathered parameters are freed
        right after it (their storage shrinks to 0 bytes) and gathered again into
        the same storage just before this unit's backward runs.  With
        ``fuse_gather_gemm`` the gather happens inside the unit's first GEMM."""
        owner = self.owner
        self._arm_grad_hooks()
        if self.fused_gather_ok(x):
            y, flat = self._forward_gathering_in_first_gemm(x)
        else:
            flat = owner._take_prefetched(self) if owner is not None else None
            flat = self.materialize(self.shard, flat)
            if owner is not None:
                owner._prefetch_after(self)
            y = self.module(x)
        if self.pg.world_size > 1 or flat.untyped_storage().data_ptr() != self.shard.untyped_storage().data_ptr():
            nbytes = flat.untyped_storage().nbytes()
            flat.untyped_storage().resize_(0)
            self._saved_flat = (flat, nbytes)
        else:
            self._saved_flat = None  # one rank: the "gathered" buffer is the shard itself
        if y.requires_grad:
            y.register_hook(self._before_backward)
        if owner is not None:
            owner._note_released(self.full_bytes)
        return y

    def _regather(self, flat: torch.Tensor, nbytes: int) -> None:
        flat.untyped_storage().resize_(nbytes)
        if self.pg.world_size > 1:
            collectives.all_gather_into(self.pg, flat, self.shard.detach())
        else:
            flat.copy_(self.shard.detach().reshape(-1))

    def _before_backward(self, grad: torch.Tensor):
        saved = self._saved_flat
        owner = self.owner
        if saved is not None:
            ready = owner._bwd_prefetched.pop(id(self), None) if owner is not None else None
            if ready is not None:
                cur = torch.cuda.current_stream(self.device)
                cur.wait_event(ready)  # gathered on the side stream
                saved[0].record_stream(cur)  # its memory is in use here until this stream is past it
            else:
                self._regather(*saved)
            if owner is not None:
                owner._note_materialized(self.full_bytes)
                owner._prefetch_backward_after(self)
        return grad

    def _arm_grad_hooks(self) -> None:
        if not getattr(self, "_hooks_installed", False):
            for p in self.params:
                p.register_post_accumulate_grad_hook(lambda _p, unit=self: unit._grad_arrived())
            self._hooks_installed = True
        self._pending = sum(1 for p in self.params if p.requires_grad)

    def _grad_arrived(self) -> None:
        self._pending -= 1
        if self._pending == 0:
            self.finish_backward()

    def finish_backward(self) -> None:
        """Reduce-scatter this unit's gradients into its shard and free everything full-size.

        On GPUs with several ranks the reduce-scatter (and the fused AdamW)
        runs on the owner's comm stream, so the next unit's backward overlaps
        it; ``sync()`` joins the comm stream back.
        """
        grads = tuple(p.grad for p in self.params)
        for p in self.params:
            p.grad = None
        owner = self.owner
        side = owner._comm_stream_for(self) if owner is not None else None
        if side is not None:
            cur = torch.cuda.current_stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                shard_grad = self.reduce_scatter_grads(grads)
            for g in grads:
                if g is not None:
                    g.record_stream(side)
            if shard_grad is not None:
                shard_grad.record_stream(cur)
        else:
            shard_grad = self.reduce_scatter_grads(grads)
        if shard_grad is not None:
            if self.shard.grad is None:
                self.shard.grad = shard_grad.view_as(self.shard)
            else:
                self.shard.grad.add_(shard_grad.view_as(self.shard))
        saved = getattr(self, "_saved_flat", None)
        if saved is not None:
            saved[0].untyped_storage().resize_(0)
            self._saved_flat = None
        self.release()
        self._pending = -1


class ShardAdamW:
    """AdamW applied to each unit's shard as part of its gradient reduce-scatter.

    Hyper-parameters live in :attr:`hp` (``lr``, ``betas``, ``eps``,
    ``weight_decay``) and are read at every step, so schedules can change
    them.  State per unit: fp32 ``m``, ``v`` and, for low-precision
    parameters, an fp32 ``master`` copy of the shard; ``step`` counts the
    unit's updates (bias correction).
    """

    def __init__(self, lr: float = 3e-4, betas: tuple[float, float] = (0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1) -> None:
        self.hp = {"lr": lr, "betas": tuple(betas), "eps": eps, "weight_decay": weight_decay}
        #: unit name -> {"step", "m", "v"[, "master"]}; names are stable across
        #: processes, so a checkpoint written by one run loads into the next.
        self.state: dict[str, dict] = {}

    def _state(self, unit: _Unit) -> dict:
        st = self.state.get(unit.name)
        if st is None:
            shard = unit.shard.detach()
            st = {"step": 0, "m": torch.zeros(shard.numel(), dtype=torch.float32, device=shard.device),
                  "v": torch.zeros(shard.numel(), dtype=torch.float32, device=shard.device)}
            if shard.dtype != torch.float32:
                st["master"] = shard.float().clone()
            self.state[unit.name] = st
        return st

    def state_dict(self) -> dict:
        """Hyper-parameters and every unit's moments, master shard and step (this rank's shards)."""
        return {"hp": dict(self.hp),
                "state": {name: {k: (v.detach().clone() if torch.is_tensor(v) else v) for k, v in st.items()}
                          for name, st in self.state.items()}}

    def load_state_dict(self, sd: dict, device: torch.device | None = None) -> None:
        self.hp = dict(sd["hp"])
        self.hp["betas"] = tuple(self.hp["betas"])
        self.state = {}
        for name, st in sd["state"].items():
            self.state[name] = {k: (v.to(device=device or v.device, dtype=torch.float32).clone().contiguous()
                                    if torch.is_tensor(v) else int(v)) for k, v in st.items()}

    @torch.no_grad()
    def step_unit(self, unit: _Unit, flat_grad: torch.Tensor) -> None:
        st = self._state(unit)
        st["step"] += 1
        W = unit.pg.world_size
        hp = self.hp
        if flat_grad.is_cuda:
            unit.pg.device_comm().reduce_scatter_adamw(
                flat_grad, unit.shard.data, st, lr=hp["lr"], betas=hp["betas"], eps=hp["eps"],
                weight_decay=hp["weight_decay"], step=st["step"], scale=1.0 / W)
            return
        g = flat_grad if W == 1 else collectives.reduce_scatter(unit.pg, flat_grad, op="sum")
        g = g.float() / W
        b1, b2 = hp["betas"]
        w = st["master"] if "master" in st else unit.shard.data
        st["m"].mul_(b1).add_(g, alpha=1 - b1)
        st["v"].mul_(b2).addcmul_(g, g, value=1 - b2)
        w.mul_(1 - hp["lr"] * hp["weight_decay"])
        denom = (st["v"] / (1 - b2 ** st["step"])).sqrt_().add_(hp["eps"])
        w.addcdiv_(st["m"] / (1 - b1 ** st["step"]), denom, value=-hp["lr"])
        if "master" in st:
            unit.shard.data.copy_(w)


class _RngSnapshot:
    """The generator states a unit's forward started from, for replaying it.

    ``capture`` records the CPU generator and, for CUDA inputs, the
    generator of that device; ``replaying()`` is a context in which both are
    back at the recorded state and after which the caller's streams continue
    exactly where they were (``fork_rng`` saves and restores them).
    """

    def __init__(self, device: torch.device) -> None:
        self.cuda_device = device if device.type == "cuda" else None
        self.cpu_state = torch.get_rng_state()
        self.cuda_state = torch.cuda.get_rng_state(device) if self.cuda_device is not None else None

    @contextlib.contextmanager
    def replaying(self):
        devices = [self.cuda_device] if self.cuda_device is not None else []
        with torch.random.fork_rng(devices=devices, enabled=True):
            torch.set_rng_state(self.cpu_state)
            if self.cuda_device is not None:
                torch.cuda.set_rng_state(self.cuda_state, self.cuda_device)
            yield


class _ShardedForward(torch.autograd.Function):
    """Unit forward with gathered parameters; backward recomputes (RNG rewound).

    Replaying the generator state is what keeps a unit with dropout correct:
    without it the recompute draws a new mask and the shard gradients are
    taken against a graph that never produced the loss, while everything
    downstream of the unit still looks fine (mini_nccl/fsdp.py:162-217).
    """

    @staticmethod
    def forward(ctx, unit: _Unit, shard: torch.Tensor, x: torch.Tensor):
        ctx.unit = unit
        ctx.save_for_backward(x, shard)
        ctx.rng = _RngSnapshot(x.device)
        owner = unit.owner
        flat = owner._take_prefetched(unit) if owner is not None else None
        with torch.no_grad():
            unit.materialize(shard, flat)
            if owner is not None:
                owner._prefetch_after(unit)
            try:
                y = unit.module(x)
            finally:
                unit.release()
        return y

    @staticmethod
    def backward(ctx, grad_y: torch.Tensor):
        x, shard = ctx.saved_tensors
        unit: _Unit = ctx.unit
        leaf = x.detach().requires_grad_(ctx.needs_input_grad[2])
        wrt = ([leaf] if leaf.requires_grad else []) + list(unit.params)
        unit.materialize(shard)
        try:
            with ctx.rng.replaying(), torch.enable_grad():
                out = unit.module(leaf)
            got = torch.autograd.grad(out, wrt, grad_outputs=grad_y, allow_unused=True)
            dx = got[0] if leaf.requires_grad else None
            shard_grad = unit.reduce_scatter_grads(got[len(wrt) - len(unit.params):])
        finally:
            unit.release()
        return None, shard_grad, dx


class _UnitWrapper(nn.Module):
    """Stands in for a sharded module inside the model tree."""

    def __init__(self, unit: _Unit) -> None:
        super().__init__()
        self.unit = unit
        self.wrapped = unit.module
        self.shard = unit.shard

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        owner = self.unit.owner
        if owner is not None and not owner.recompute and torch.is_grad_enabled():
            return self.unit.forward_saving_activations(x)
        return _ShardedForward.apply(self.unit, self.shard, x)


class FullyShardedDataParallel(nn.Module):
    """Shard every ``unit_cls`` child (or each module in ``units``) across ``pg``."""

    def __init__(
        self,
        module: nn.Module,
        pg: Communicator,
        unit_cls: type | tuple[type, ...] | None = None,
        units: list[nn.Module] | None = None,
        prefetch: bool = False,
        optimizer_in_backward: dict | None = None,
        recompute: bool = True,
        fuse_gather_gemm: bool = False,
    ) -> None:
        super().__init__()
        if unit_cls is None and units is None:
            raise ValueError("pass unit_cls or units to say what should be sharded")
        if fuse_gather_gemm and recompute:
            raise ValueError("fuse_gather_gemm needs recompute=False (activations kept)")
        #: Gather each unit's parameters inside its first GEMM (one kernel;
        #: units that provide ``fsdp_forward_with_gathered_gemm``).  Units then
        #: keep their 1-D parameters whole on every rank (averaged in ``sync``).
        self.fuse_gather_gemm = fuse_gather_gemm
        self.pg = pg
        self.shard_optimizer = ShardAdamW(**optimizer_in_backward) if optimizer_in_backward is not None else None
        self.recompute = recompute
        self.units: list[_Unit] = []
        self._live_bytes = 0
        self.peak_materialized_bytes = 0
        self.prefetch = prefetch
        self._prefetched: dict[int, tuple[torch.Tensor, torch.cuda.Event]] = {}
        self._param_names = {id(p): name for name, p in module.named_parameters()}

        if pg.world_size > 1:
            with torch.no_grad():
                for p in module.parameters():
                    collectives.broadcast(pg, p.data, src=0)
                for b in module.buffers():
                    collectives.broadcast(pg, b.data, src=0)

        chosen = {id(m) for m in (units or [])}
        for parent in list(module.modules()):
            for key, child in list(parent._modules.items()):
                if child is None:
                    continue
                hit = id(child) in chosen or (unit_cls is not None and isinstance(child, unit_cls))
                if not hit or not any(True for _ in child.parameters()):
                    continue
                unit = _Unit(child, pg, name=f"{type(child).__name__.lower()}{len(self.units)}",
                             keep_vectors_whole=fuse_gather_gemm)
                unit.owner = self
                self.units.append(unit)
                parent._modules[key] = _UnitWrapper(unit)
        if not self.units:
            raise ValueError("no modules matched unit_cls/units, so nothing would be sharded")

        self.module = module
        unit_ids = {id(p) for u in self.units for p in u.params}
        shard_ids = {id(u.shard) for u in self.units}
        self._replicated = [
            p for p in module.parameters() if id(p) not in unit_ids and id(p) not in shard_ids
        ]
        self._index = {id(u): i for i, u in enumerate(self.units)}
        self._side = None
        self._comm_stream = None
        self._bwd_prefetched: dict[int, torch.cuda.Event] = {}
        # Two gradient buffers in NVLS memory, used by turns in unit order (the
        # same on every rank).  Two, because a rank may flatten the next unit
        # while a slower rank's switch reads of the previous one still run; the
        # reduce-scatter of unit i+1 starts only once every rank has entered it,
        # i.e. has finished unit i, so buffer i % 2 is free again by then.
        self._grad_bufs: list[torch.Tensor] | None = None
        self._grad_turn = 0
        dev = self.units[0].device
        if FSDP_NVLS_GRADS and dev.type == "cuda" and pg.world_size > 1:
            dc = pg.device_comm()
            if dc.nvls:
                nbytes = max(u.padded_numel * u.shard.element_size() for u in self.units)
                nbytes = -(-nbytes // 16) * 16  # any unit dtype views it whole
                self._grad_bufs = [dc.symmetric_zeros(nbytes, torch.uint8, nvls=True) for _ in range(2)]

    def _grad_buffer(self, unit: _Unit) -> torch.Tensor | None:
        """The next NVLS gradient buffer, as ``unit.padded_numel`` of its dtype (or None)."""
        if self._grad_bufs is None:
            return None
        buf = self._grad_bufs[self._grad_turn]
        self._grad_turn ^= 1
        return buf.view(unit.dtype)[: unit.padded_numel]

    # ---- prefetch (CUDA) -----------------------------------------------------------

    def _prefetch_after(self, unit: _Unit) -> None:
        if not self.prefetch or unit.device.type != "cuda" or self.pg.world_size == 1:
            return
        if self.fuse_gather_gemm:  # the next unit gathers inside its own first GEMM
            return
        i = self._index[id(unit)] + 1
        if i >= len(self.units) or i in self._prefetched:
            return
        nxt = self.units[i]
        if self._side is None:
            self._side = torch.cuda.Stream(device=unit.device)
        cur = torch.cuda.current_stream(unit.device)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            flat = nxt._gather(nxt.shard)
            done = torch.cuda.Event()
            done.record(self._side)
        flat.record_stream(cur)
        self._prefetched[i] = (flat, done)

    def _prefetch_backward_after(self, unit: _Unit) -> None:
        """Gather the unit whose backward comes next (the previous one) on the side stream."""
        if not self.prefetch or unit.device.type != "cuda" or self.pg.world_size == 1:
            return
        i = self._index[id(unit)] - 1
        if i < 0:
            return
        prev = self.units[i]
        saved = getattr(prev, "_saved_flat", None)
        if saved is None or id(prev) in self._bwd_prefetched:
            return
        if self._side is None:
            self._side = torch.cuda.Stream(device=unit.device)
        cur = torch.cuda.current_stream(unit.device)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            prev._regather(*saved)
            done = torch.cuda.Event()
            done.record(self._side)
        self._bwd_prefetched[id(prev)] = done

    def _comm_stream_for(self, unit: _Unit):
        if unit.device.type != "cuda" or self.pg.world_size == 1 or self.recompute:
            return None
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device=unit.device)
        return self._comm_stream

    def _take_prefetched(self, unit: _Unit):
        hit = self._prefetched.pop(self._index[id(unit)], None)
        if hit is None:
            return None
        flat, done = hit
        torch.cuda.current_stream(unit.device).wait_event(done)
        return flat

    # ---- what the optimizer sees ------------------------------------------------------

    def shard_parameters(self) -> list[nn.Parameter]:
        return [u.shard for u in self.units]

    def replicated_parameters(self) -> list[nn.Parameter]:
        """Parameters outside every unit (kept whole on each rank, averaged in ``sync``).

        With ``optimizer_in_backward`` these are all the user's optimizer has
        to step: the shards are updated inside the reduce-scatter."""
        return list(self._replicated)

    def parameters(self, recurse: bool = True):
        """Shards and replicated parameters only (never the transient full ones)."""
        return iter(self.shard_parameters() + self._replicated)

    def named_parameters(
        self, prefix: str = "", recurse: bool = True, remove_duplicate: bool = True
    ) -> Iterator[tuple[str, nn.Parameter]]:
        for u in self.units:
            yield f"{prefix}{u.name}.shard", u.shard
        for p in self._replicated:
            yield prefix + self._param_names.get(id(p), "replicated"), p

    # ---- memory accounting --------------------------------------------------------------

    def _note_materialized(self, nbytes: int) -> None:
        self._live_bytes += nbytes
        self.peak_materialized_bytes = max(self.peak_materialized_bytes, self._live_bytes)

    def _note_released(self, nbytes: int) -> None:
        self._live_bytes = max(0, self._live_bytes - nbytes)

    def memory_report(self) -> dict[str, int]:
        """Measured bytes of parameter storage per rank."""
        item = self.units[0].shard.element_size()
        full = sum(u.padded_numel for u in self.units) * item
        resident = sum(u.shard_numel for u in self.units) * item
        replicated = sum(p.numel() * p.element_size() for p in self._replicated)
        return {
            "sharded_params_full": full,
            "sharded_params_resident": resident,
            "replicated_params": replicated,
            "peak_transient": self.peak_materialized_bytes,
            "ddp_equivalent": full + replicated,
            "fsdp_peak": resident + replicated + self.peak_materialized_bytes,
        }

    # ---- training ----------------------------------------------------------------------------

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def sync(self) -> None:
        """Average the replicated gradients (sharded ones were done in backward)."""
        for u in self.units:  # units whose parameters did not all receive gradients
            if getattr(u, "_pending", -1) > 0:
                u.finish_backward()
        if self._comm_stream is not None:  # shard gradients / updates made on the comm stream
            torch.cuda.current_stream(self._comm_stream.device).wait_stream(self._comm_stream)
        if self.pg.world_size == 1 or not self._replicated:
            return
        average_gradients(self.pg, self._replicated)

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.parameters():
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    # ---- checkpointing -------------------------------------------------------------------------

    def full_state_dict(self) -> dict[str, torch.Tensor]:
        """The unsharded model under its original parameter names."""
        state: dict[str, torch.Tensor] = {}
        for u in self.units:
            flat = u.gather_full_flat()
            at = 0
            for p, (_, _, shape, n) in zip(u.params, u.entries, strict=True):
                name = self._param_names.get(id(p), f"{u.name}.{at}")
                state[name] = flat[at : at + n].view(shape).clone()
                at += n
        for p in self._replicated:
            name = self._param_names.get(id(p))
            if name is not None:
                state[name] = p.detach().clone()
        for name, b in self.module.named_buffers():
            state[name] = b.detach().clone()
        return state

    def sharded_state_dict(self, optimizer: torch.optim.Optimizer | None = None) -> dict[str, object]:
        """Everything this rank needs to resume, as one per-rank checkpoint.

        Holds this rank's shards, the replicated parameters and buffers, the
        fused shard optimizer's state (fp32 master shards, moments and step
        counts) when ``optimizer_in_backward`` is on, and the ``state_dict`` of
        ``optimizer`` (the user's optimizer over shards and replicated
        parameters) when given.  Save it with ``torch.save`` to one file per
        rank; :meth:`load_sharded_state_dict` restores it on the same layout,
        after which training continues bit for bit as if never interrupted.
        """
        sd: dict[str, object] = {
            "rank": self.pg.rank,
            "world_size": self.pg.world_size,
            "shards": {u.name: u.shard.detach().clone() for u in self.units},
            "replicated": {
                self._param_names.get(id(p), f"replicated{i}"): p.detach().clone()
                for i, p in enumerate(self._replicated)
            },
            "buffers": {name: b.detach().clone() for name, b in self.module.named_buffers()},
        }
        if self.shard_optimizer is not None:
            sd["shard_optimizer"] = self.shard_optimizer.state_dict()
        if optimizer is not None:
            sd["optimizer"] = optimizer.state_dict()
        return sd

    def load_sharded_state_dict(self, state: dict[str, object],
                                optimizer: torch.optim.Optimizer | None = None) -> None:
        if state["world_size"] != self.pg.world_size or state["rank"] != self.pg.rank:
            raise ValueError("sharded checkpoint was written by a different rank layout")
        shards = state["shards"]
        replicated = state["replicated"]
        with torch.no_grad():
            for u in self.units:
                u.shard.copy_(shards[u.name])  # type: ignore[index]
            for i, p in enumerate(self._replicated):
                p.copy_(replicated[self._param_names.get(id(p), f"replicated{i}")])  # type: ignore[index]
            for name, b in self.module.named_buffers():
                saved = state.get("buffers", {}).get(name)  # type: ignore[union-attr]
                if saved is not None:
                    b.copy_(saved)
        if self.shard_optimizer is not None and "shard_optimizer" in state:
            device = self.units[0].shard.device
            self.shard_optimizer.load_state_dict(state["shard_optimizer"], device=device)  # type: ignore[arg-type]
        if optimizer is not None:
            if "optimizer" not in state:
                raise ValueError("the checkpoint holds no optimizer state")
            optimizer.load_state_dict(state["optimizer"])  # type: ignore[arg-type]
