"""Host-side failure detection for multi-rank serving.

Every rank publishes a heartbeat (step counter and wall time) to the
process-group store after each engine step. Before a rank enters the next
collective it checks that every peer's heartbeat is fresh; a peer that stopped
beating (crashed, hung in Python, or left between steps) is reported as a
:class:`PeerFailure` instead of leaving this rank blocked inside NCCL. Process
groups are created with a short timeout as the second line of defence, and
device-side waits are bounded in the kernels themselves (kErrPeerWait).
"""
from __future__ import annotations

import time


class PeerFailure(RuntimeError):
    def __init__(self, ranks: list[int], detail: str = ""):
        super().__init__(f"peer rank(s) {ranks} stopped responding{': ' + detail if detail else ''}")
        self.ranks = ranks


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "gsb/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.step = 0
        self.beat()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.step += 1
        self.store.set(self._key(self.rank), f"{self.step}:{time.time():.6f}")

    def leave(self) -> None:
        """Announce an orderly exit (peers then fail fast instead of waiting out the timeout)."""
        self.store.set(self._key(self.rank), f"-1:{time.time():.6f}")

    def peers_status(self) -> dict[int, tuple[int, float]]:
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                v = self.store.get(self._key(r)).decode()
                s, t = v.split(":")
                out[r] = (int(s), float(t))
            except Exception:
                out[r] = (0, 0.0)
        return out

    def check(self) -> None:
        """Raise :class:`PeerFailure` if a peer left or has not beaten within the timeout."""
        now = time.time()
        bad, why = [], []
        for r, (step, t) in self.peers_status().items():
            if step < 0:
                bad.append(r)
                why.append(f"rank {r} left")
            elif now - t > self.timeout_s:
                bad.append(r)
                why.append(f"rank {r} silent for {now - t:.1f}s")
        if bad:
            raise PeerFailure(bad, "; ".join(why))
