"""The producer side's ledger of prefill blocks held for decode readers.

A prefill rank keeps a handed-over request's blocks until every decode rank that reads from it has said its copy
landed, or until the abort timeout passes -- a pull is one-sided, so the producer cannot see one in flight, and the
timeout is long for that. Those are the reference's rules (lean_vllm/kv_transfer/nixl_connector.py:257-306):

* a request is held from hand-over (the scheduler's reqs_to_send) until a deadline;
* each reader's notification names how many readers the request has (the "request:readers" message);
* the request is released once that many have reported -- whether they report before or after the hand-over;
* a held request past its deadline is released as expired;
* notifications for a request never handed over here are forgotten once they are older than the timeout.

The ledger only keeps the books; the worker turns its answers into finished_sending / expired_sending under its
own lock.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(slots=True)
class _Tally:
    reported: int  # notifications received
    readers: int  # how many the request has, as its notifications say
    first: float  # monotonic time of the first


class Holds:
    def __init__(self):
        self._deadlines: dict[str, float] = {}  # held request -> when it expires
        self._tallies: dict[str, _Tally] = {}  # request -> its readers' reports so far, held or not

    def __contains__(self, request_id: str) -> bool:
        return request_id in self._deadlines

    def hold(self, request_id: str, deadline: float) -> bool:
        """Holds a handed-over request's blocks until `deadline`. True if every reader has reported already, in
        which case the request is not held and its blocks go back now."""
        self._deadlines[request_id] = deadline
        return self._complete(request_id)

    def reported(self, request_id: str, readers: int, now: float) -> bool:
        """One reader's copy landed. True if that was the last reader of a held request, which is then let go."""
        tally = self._tallies.get(request_id)
        if tally is None:
            tally = self._tallies[request_id] = _Tally(0, readers, now)
        tally.reported += 1
        return self._complete(request_id)

    def expire(self, now: float) -> list[str]:
        """Held requests past their deadline, let go."""
        overdue = [request_id for request_id, deadline in self._deadlines.items() if deadline < now]
        for request_id in overdue:
            self._let_go(request_id)
        return overdue

    def forget_strays(self, now: float, timeout: float) -> None:
        """Drops reports older than `timeout` for requests never held here (not this engine's hand-over)."""
        stale = [request_id for request_id, tally in self._tallies.items()
                 if request_id not in self._deadlines and tally.first + timeout < now]
        for request_id in stale:
            del self._tallies[request_id]

    def _complete(self, request_id: str) -> bool:
        tally = self._tallies.get(request_id)
        if request_id not in self._deadlines or tally is None or tally.reported < tally.readers:
            return False
        self._let_go(request_id)
        return True

    def _let_go(self, request_id: str) -> None:
        del self._deadlines[request_id]
        self._tallies.pop(request_id, None)
