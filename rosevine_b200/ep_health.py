"""Failure handling of the expert-parallel ranks: bounded communicator set-up, a host-side
liveness check before every step's exchanges, and abort.

A rank of the expert-parallel layer (rosevine_b200.ep) only leaves between steps, with none of
its kernels or collectives in flight. The others must learn of it before they enter the next
step's all-to-all, which would otherwise wait on the missing peer: the reference's CPU expert
pool has the same contract for its workers (runtime/src/expert_pool.rs: a worker that fails is
reported to the caller as an error and the pool stays usable, never a hang).

- init_ep_group: the process group with a short timeout; on NCCL the communicators are created
  non-blocking (NCCL config blocking = 0) and eagerly for this rank's device, so a peer that
  never joins ends the set-up with an error after the timeout instead of blocking it.
- EpHealth: before each step every rank publishes "step s reached" in the group's key-value
  store and waits, bounded, until every peer has published it. A peer that announced its exit
  (leave()) is reported at once; one that stalls is reported when the timeout runs out. Either
  way the step raises PeerLost before any collective of that step is issued, and the raising
  rank leaves too, so that a peer that comes back late learns of it instead of waiting. The
  healthy path costs two store round trips per step.
- A store that can no longer be reached (the rank hosting it has exited) is reported the same
  way, as PeerLost("unreachable").
- abort_ep_group: tears the group down without waiting for peers (ncclCommAbort under NCCL).

The process-group timeout stays the last bound for a failure the liveness check cannot see (a
rank that dies inside a step): the next collective then ends with an error.
"""
from __future__ import annotations

import time
from datetime import timedelta

import torch
import torch.distributed as dist


class PeerLost(RuntimeError):
    """Some ranks did not reach a step: `ranks` that left or stalled, `why` ("left" or "timeout")."""

    def __init__(self, ranks, why: str, step: int):
        self.ranks, self.why, self.step = list(ranks), why, step
        super().__init__(f"expert-parallel step {step}: ranks {self.ranks} {why}")


def init_ep_group(backend: str, rank: int, world: int, timeout_s: float = 30.0, device: int | None = None,
                  store=None) -> None:
    """torch.distributed process group for the expert-parallel layer, set up with a bound.
    MASTER_ADDR / MASTER_PORT (or `store`) as for init_process_group."""
    kw = {"backend": backend, "rank": rank, "world_size": world, "timeout": timedelta(seconds=timeout_s)}
    if store is not None:
        kw["store"] = store
    if backend == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.blocking = 0  # non-blocking communicator set-up: errors surface, nothing hangs
        kw["pg_options"] = opts
        kw["device_id"] = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    dist.init_process_group(**kw)


def abort_ep_group() -> None:
    """End the default process group without a rendezvous with the peers."""
    if not dist.is_initialized():
        return
    abort = getattr(dist.distributed_c10d, "_abort_process_group", None)
    if abort is not None and dist.get_backend() == "nccl":
        abort()
    else:
        dist.destroy_process_group()


class EpHealth:
    """Per-step liveness of the ranks through the process group's key-value store."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, poll_s: float = 0.002,
                 prefix: str = "ep"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.poll_s, self.prefix = timeout_s, poll_s, prefix

    def _key(self, step: int, r: int) -> str:
        return f"{self.prefix}/step{step}/{r}"

    def _left(self, r: int) -> str:
        return f"{self.prefix}/left/{r}"

    def begin_step(self, step: int) -> None:
        """Publish that this rank reached `step`; return once every peer has, else raise PeerLost
        (why "unreachable" when the store itself is gone: its host rank has exited)."""
        try:
            self._begin_step(step)
        except PeerLost:
            raise
        except Exception as e:  # noqa: BLE001 - the store's connection errors vary by backend
            raise PeerLost([r for r in range(self.world) if r != self.rank], "unreachable", step) from e

    def _begin_step(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), b"1")
        if step >= 2:  # this rank's older marks are no longer read by anyone
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except Exception:  # noqa: BLE001 - a store without deletion keeps them
                pass
        peers = [r for r in range(self.world) if r != self.rank]
        keys = [self._key(step, r) for r in peers]
        deadline = time.monotonic() + self.timeout_s
        while True:
            # fast path, two store round trips: every peer's mark is there and nobody has left (a
            # peer that reached the step and then gave up on it has left: no exchange of this
            # step would complete)
            present = self.store.check(keys)
            n_left = self.store.add(self._nleft(), 0)
            if present and n_left == 0:
                return
            if n_left:
                left = [r for r in peers if self.store.check([self._left(r)])]
                if left:
                    # a peer that gave up on a stalled rank names it: every healthy rank then
                    # reports the same cause, whichever of them ran out of time first
                    stalled = sorted({s for r in left for s in self._stalled(r)} - {self.rank})
                    if stalled and not any(self.rank in self._stalled(r) for r in left):
                        self.leave(stalled)
                        raise PeerLost(stalled, "timeout", step)
                    self.leave()
                    raise PeerLost(left, "left", step)
            if time.monotonic() > deadline:
                missing = [r for r in peers if not self.store.check([self._key(step, r)])]
                self.leave(missing)
                raise PeerLost(missing, "timeout", step)
            time.sleep(self.poll_s)

    def _nleft(self) -> str:
        return f"{self.prefix}/n_left"

    def _stalled(self, r: int) -> list[int]:
        """The ranks that peer r gave up waiting on when it left (empty: it left of its own accord)."""
        v = self.store.get(self._left(r)).decode()
        return [int(t) for t in v[2:].split(",")] if v.startswith("t:") else []

    def leave(self, stalled=()) -> None:
        """Announce that this rank takes no further steps (between steps; begin_step does it
        itself before raising PeerLost, naming the ranks it timed out on). Idempotent."""
        try:
            if not self.store.check([self._left(self.rank)]):
                mark = "t:" + ",".join(str(r) for r in stalled) if stalled else "x"
                self.store.set(self._left(self.rank), mark.encode())
                self.store.add(self._nleft(), 1)
        except Exception:  # noqa: BLE001 - nobody is left to tell
            pass
