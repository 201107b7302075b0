"""The producer's ledger of held prefill blocks (kv_transfer/holds.py) against the reference's release rules
(lean_vllm/kv_transfer/nixl_connector.py:257-306): release when as many readers as the notifications name have
reported, before or after the hand-over; expire at the deadline; forget reports for requests never handed over."""

from lean_vllm_b200.kv_transfer.holds import Holds


def test_a_request_is_released_when_its_last_reader_reports():
    holds = Holds()
    assert holds.hold("r", deadline=100.0) is False
    assert holds.reported("r", readers=2, now=1.0) is False
    assert "r" in holds
    assert holds.reported("r", readers=2, now=2.0) is True
    assert "r" not in holds


def test_readers_that_report_before_the_hand_over_release_it_at_the_hand_over():
    holds = Holds()
    assert holds.reported("r", readers=1, now=1.0) is False  # not held yet: kept
    assert holds.hold("r", deadline=100.0) is True
    assert "r" not in holds


def test_a_held_request_expires_at_its_deadline_and_only_then():
    holds = Holds()
    holds.hold("a", deadline=10.0)
    holds.hold("b", deadline=20.0)
    holds.reported("a", readers=2, now=1.0)
    assert holds.expire(now=5.0) == []
    assert holds.expire(now=15.0) == ["a"]
    assert "a" not in holds and "b" in holds
    assert holds.reported("a", readers=2, now=16.0) is False  # a late reader of an expired request changes nothing


def test_reports_for_a_request_never_handed_over_are_forgotten_after_the_timeout():
    holds = Holds()
    holds.reported("stray", readers=3, now=0.0)
    holds.forget_strays(now=5.0, timeout=10.0)
    holds.hold("stray", deadline=100.0)
    assert holds.reported("stray", readers=3, now=6.0) is False
    assert holds.reported("stray", readers=3, now=6.0) is True  # kept: 3 reports in all
    holds2 = Holds()
    holds2.reported("stray", readers=1, now=0.0)
    holds2.forget_strays(now=11.0, timeout=10.0)
    assert holds2.hold("stray", deadline=100.0) is False  # forgotten: the hand-over waits for a new report
