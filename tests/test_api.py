"""The connector API's shared pieces (reference tests/test_kv_transfer.py:87-189) and the scheduler half
(nixl_connector.py:111-168), on the package's own classes."""

from dataclasses import dataclass, field

import pytest

from lean_vllm_b200.kv_transfer import (
    CONNECTORS,
    KVConnectorMetadata,
    KVConnectorOutput,
    KVOutputAggregator,
    KVTransferConfig,
    KVTransferStats,
    check_kv_transfer_params,
    create_scheduler_connector,
    parse_kv_transfer_config,
)
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler


class TestAggregator:
    def test_a_transfer_finishes_once_every_rank_reports_it(self):
        aggregator = KVOutputAggregator(world_size=2)
        assert not aggregator.aggregate([KVConnectorOutput(finished_recving={"a"}), KVConnectorOutput()])
        result = aggregator.aggregate([KVConnectorOutput(), KVConnectorOutput(finished_recving={"a"})])
        assert result == KVConnectorOutput(finished_recving={"a"})

    def test_one_rank_failing_fails_the_load(self):
        aggregator = KVOutputAggregator(world_size=2)
        result = aggregator.aggregate(
            [KVConnectorOutput(failed_recving={"a"}), KVConnectorOutput(finished_recving={"a"})])
        assert result == KVConnectorOutput(failed_recving={"a"})

    def test_sends_count_the_same_way(self):
        aggregator = KVOutputAggregator(world_size=2)
        assert not aggregator.aggregate([KVConnectorOutput(finished_sending={"a"}), KVConnectorOutput()])
        done = aggregator.aggregate([KVConnectorOutput(), KVConnectorOutput(finished_sending={"a"})])
        assert done.finished_sending == {"a"}

    def test_a_load_s_stats_take_the_slowest_rank_and_every_rank_s_bytes(self):
        aggregator = KVOutputAggregator(world_size=2)
        result = aggregator.aggregate([
            KVConnectorOutput(finished_recving={"a"}, recv_stats={"a": KVTransferStats(0.1, 100)}),
            KVConnectorOutput(finished_recving={"a"}, recv_stats={"a": KVTransferStats(0.3, 100)}),
        ])
        assert result.recv_stats == {"a": KVTransferStats(0.3, 200)}

    def test_a_failed_load_has_no_stats(self):
        aggregator = KVOutputAggregator(world_size=2)
        result = aggregator.aggregate([
            KVConnectorOutput(failed_recving={"a"}),
            KVConnectorOutput(finished_recving={"a"}, recv_stats={"a": KVTransferStats(0.3, 100)}),
        ])
        assert result.failed_recving == {"a"} and result.recv_stats == {}

    def test_an_expiry_on_any_rank_counts_once(self):
        aggregator = KVOutputAggregator(world_size=2)
        aggregator.aggregate([KVConnectorOutput(finished_sending={"a"}, expired_sending={"a"}), KVConnectorOutput()])
        result = aggregator.aggregate([KVConnectorOutput(), KVConnectorOutput(finished_sending={"a"})])
        assert result.expired_sending == {"a"}

    def test_the_reference_s_own_output_objects_aggregate_too(self):
        """Duck-typed: the aggregator reads attributes only, so it takes any object of the same fields."""

        @dataclass
        class Foreign:
            finished_sending: set = field(default_factory=set)
            finished_recving: set = field(default_factory=set)
            failed_recving: set = field(default_factory=set)
            expired_sending: set = field(default_factory=set)
            recv_stats: dict = field(default_factory=dict)

        assert KVOutputAggregator(1).aggregate([Foreign(finished_recving={"x"})]).finished_recving == {"x"}


class TestConfig:
    def test_the_json_flag_parses(self):
        kv = parse_kv_transfer_config('{"kv_role": "kv_consumer", "kv_port": 15000}')
        assert (kv.kv_connector, kv.kv_role, kv.kv_port) == ("CudaIpcConnector", "kv_consumer", 15000)
        assert kv.is_consumer and not kv.is_producer

    @pytest.mark.parametrize(
        "value, message",
        [
            ('{"kv_role": "decoder"}', "kv_role\n  Input should be 'kv_producer'"),
            ('{"kv_connector": "MooncakeConnector"}', "unknown kv_connector"),
            ('{"kv_buffer_size": 1}', "kv_buffer_size\n  Unexpected keyword argument"),
        ],
    )
    def test_a_bad_flag_is_named(self, value, message):
        with pytest.raises(ValueError, match=message):
            parse_kv_transfer_config(value)

    def test_each_engine_gets_its_own_id(self):
        assert parse_kv_transfer_config("{}").engine_id != parse_kv_transfer_config("{}").engine_id

    def test_the_factory_builds_the_scheduler_half(self):
        @dataclass
        class Config:
            kv_transfer: KVTransferConfig
            kvcache_block_size: int = 16
            tensor_parallel_size: int = 1

        assert isinstance(create_scheduler_connector(Config(KVTransferConfig())), CudaIpcConnectorScheduler)
        assert set(CONNECTORS) == {"CudaIpcConnector"}


class TestRequestParams:
    BOTH = KVTransferConfig(kv_role="kv_both")
    PULL = dict(do_remote_prefill=True, remote_block_ids=[1], remote_request_id="p", remote_engine_id="e",
                remote_host="h", remote_port=1)

    def test_well_formed_params_pass(self):
        assert check_kv_transfer_params({"do_remote_decode": True}, self.BOTH) is None
        assert check_kv_transfer_params(self.PULL, self.BOTH) is None

    @pytest.mark.parametrize(
        "params, kv_role, message",
        [
            ({"do_remote_decode": True}, None, "needs an engine started with kv_transfer_config"),
            ({"do_remote_decode": True}, "kv_consumer", "do_remote_decode needs kv_role"),
            (PULL, "kv_producer", "do_remote_prefill needs kv_role"),
            (PULL | {"remote_port": "1"}, "kv_both", "remote_port: Input should be a valid integer"),
            (PULL | {"remote_block_ids": ["x"]}, "kv_both", "remote_block_ids.0: Input should be a valid integer"),
            ({k: v for k, v in PULL.items() if k != "remote_host"}, "kv_both", "remote_host: Field required"),
            ([1], "kv_both", "must be an object"),
        ],
    )
    def test_what_the_engine_cannot_honour_is_named(self, params, kv_role, message):
        kv = KVTransferConfig(kv_role=kv_role) if kv_role else None
        assert message in check_kv_transfer_params(params, kv)


@dataclass
class FakeSeq:
    """The Sequence fields the scheduler half reads."""

    request_id: str
    num_prompt_tokens: int
    block_table: list
    kv_transfer_params: dict | None = None
    num_cached_tokens: int = 0
    finish_reason: str | None = None


@dataclass
class SchedConfig:
    kv_transfer: KVTransferConfig
    kvcache_block_size: int = 16
    tensor_parallel_size: int = 2


class TestSchedulerHalf:
    def half(self):
        return CudaIpcConnectorScheduler(SchedConfig(KVTransferConfig(engine_id="pre", kv_ip="10.0.0.1",
                                                                      kv_port=15000)))

    def params(self, blocks):
        return dict(do_remote_prefill=True, remote_block_ids=blocks, remote_request_id="p-1",
                    remote_engine_id="pre", remote_host="10.0.0.1", remote_port=15000, tp_size=2)

    def test_a_prefill_that_ran_to_its_token_hands_over_its_prompt_blocks(self):
        half = self.half()
        seq = FakeSeq("p-1", 40, [7, 3, 9, 1], {"do_remote_decode": True}, finish_reason="length")
        hold, params = half.request_finished(seq)
        assert hold and params == dict(do_remote_prefill=True, do_remote_decode=False, remote_request_id="p-1",
                                       remote_engine_id="pre", remote_block_ids=[7, 3, 9], remote_host="10.0.0.1",
                                       remote_port=15000, tp_size=2)
        assert half.build_connector_meta() == KVConnectorMetadata(reqs_to_send={"p-1": [7, 3, 9]})
        assert not half.build_connector_meta()

    @pytest.mark.parametrize("reason", ["abort", None])
    def test_an_aborted_prefill_or_a_plain_request_hands_nothing_over(self, reason):
        half = self.half()
        assert half.request_finished(FakeSeq("p", 40, [1, 2, 3], {"do_remote_decode": True},
                                             finish_reason=reason)) == (False, None)
        assert half.request_finished(FakeSeq("q", 40, [1, 2, 3], None, finish_reason="stop")) == (False, None)

    def test_a_decode_request_loads_every_token_past_the_local_hits(self):
        half = self.half()
        seq = FakeSeq("d-1", 40, [], self.params([7, 3, 9]))
        assert half.get_num_new_matched_tokens(seq, 16) == (24, True)

    def test_a_block_count_that_does_not_fit_the_prompt_prefills_here(self, caplog):
        half = self.half()
        seq = FakeSeq("d-1", 40, [], self.params([7, 3]))
        assert half.get_num_new_matched_tokens(seq, 0) == (0, False)
        assert seq.kv_transfer_params["do_remote_prefill"] is False
        assert "2 remote blocks for a 3-block prompt" in caplog.text

    def test_the_load_skips_blocks_cached_here_and_happens_once(self):
        half = self.half()
        seq = FakeSeq("d-1", 40, [20, 21, 22], self.params([7, 3, 9]), num_cached_tokens=16)
        half.update_state_after_alloc(seq, 24)
        meta = half.build_connector_meta()
        req = meta.reqs_to_recv["d-1"]
        assert (req.local_block_ids, req.remote_block_ids, req.remote_tp_size) == ([21, 22], [3, 9], 2)
        assert seq.kv_transfer_params["do_remote_prefill"] is False  # a preempted request recomputes
        assert half.get_num_new_matched_tokens(seq, 0) == (0, False)
