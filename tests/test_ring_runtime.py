"""Ring runtime rank plans (C++): geometry validation, DSA candidate buckets,
execution-row capacity, endpoint capability profiles, the pure-pipeline and TP x PP
builders, and agreement of every rank's plan in a ring.

Behaviour follows crates/spark-node/src/rank_daemon/ring_runtime.rs (geometry
:222-300, validate_endpoint :378-414, build_rank_plan / build_shape_rank_plan)."""
import pytest

from sparkpipe_rs_b200.core import core

C = core()
R, TP = C.ring_runtime, C.tp


def geometry(stages=(4, 8, 8, 8), gpus_per_node=2, first_routed=1):
    g = R.Geometry()
    g.layer_count = sum(stages)
    g.first_routed_layer = first_routed
    g.hidden_dimension = 2048
    g.maximum_context_tokens = 131072
    g.dsa_selected_tokens = 2048
    g.dsa_index_bytes_per_sequence = 2048 * 4
    g.max_speculative_rows_per_lane = 4
    g.max_batch_bucket = 1024
    g.stage_count = len(stages)
    g.default_stage_layer_counts = list(stages)
    g.host_prefix = "b200-"
    g.gpus_per_node = gpus_per_node
    g.tp_geometry = TP.Geometry(16, 192, 256, 128)
    g.shape_inputs = TP.ModelInputs(sum(stages), 2048, 1408, 10944, 576)
    return g


def test_geometry_helpers():
    g = geometry()
    g.validate()
    assert [R.dsa_candidate_bucket(g, n) for n in (0, 1, 2048, 2049, 5000, 131072, 131073)] == [
        0, 2048, 2048, 4096, 8192, 131072, 0]
    assert [R.execution_row_capacity(g, n) for n in (0, 1, 64, 256, 1024, 1025)] == [0, 4, 256, 1024, 1024, 0]
    assert R.rank_host_name(g, 0) == "b200-0" and R.rank_host_name(g, 3) == "b200-1"
    bad = geometry()
    bad.default_stage_layer_counts = [4, 8, 8, 7]
    with pytest.raises(Exception):
        bad.validate()


def test_endpoint_profiles():
    e = R.Endpoint()
    e.transport, e.route_name = "nvlink.peer_memory", "a_to_b_hidden"
    e.hidden_dimension, e.bytes_per_sequence, e.max_active_sequences, e.max_packet_bytes = 2048, 4096, 8, 8 * 4096
    for caps in (R.CAPS_PEER_PRODUCTION, R.CAPS_HOST_STAGED, R.CAPS_SIMULATION):
        e.capability_flags = caps
        R.validate_endpoint(e)
    for caps in (R.CAPS_PEER_PRODUCTION & ~0x4, R.CAPS_SIMULATION | R.CAPS_PEER_PRODUCTION, 0):
        e.capability_flags = caps
        with pytest.raises(Exception):
            R.validate_endpoint(e)
    e.capability_flags = R.CAPS_HOST_STAGED
    e.max_packet_bytes = 100  # below one row per sequence
    with pytest.raises(Exception):
        R.validate_endpoint(e)


def test_pipeline_plans():
    g = geometry()
    plans = R.build_ring(g, 1, 64)
    assert [(p.first_layer, p.layer_count) for p in plans] == [(0, 4), (4, 8), (12, 8), (20, 8)]
    p0, p1, p2, p3 = plans
    assert p0.flags == R.FLAG_HAS_NEXT | R.FLAG_DENSE_PREFIX and p0.previous_rank == R.NO_RANK
    assert p3.flags == R.FLAG_HAS_PREVIOUS | R.FLAG_FINAL_STAGE and p3.next_rank == R.NO_RANK
    assert p1.previous_rank == 0 and p1.next_rank == 2 and p1.listen_port == R.DEFAULT_PORT_BASE + 1
    assert p1.next_port == R.DEFAULT_PORT_BASE + 2 and p0.output_route == p1.input_route
    # ranks 0,1 share node b200-0: NVLink peer memory; rank 1 -> 2 crosses nodes: host staged
    assert p0.output_endpoint.transport == "nvlink.peer_memory"
    assert p0.output_endpoint.capability_flags == R.CAPS_PEER_PRODUCTION
    assert p1.output_endpoint.transport == "fabric.host_staged_tcp" and p2.host == "b200-1"
    assert p1.execution_row_capacity == 256 and p1.max_packet_bytes == 256 * (4096 + 8192)
    assert p3.final_event_host == "b200-0" and p3.final_event_port == R.DEFAULT_PORT_BASE + R.FINAL_EVENT_PORT_OFFSET
    assert p3.final_event_route and not p1.final_event_route
    with pytest.raises(Exception):
        R.build_rank_plan(g, 4, 64)  # no such stage
    with pytest.raises(Exception):
        R.build_rank_plan(g, 0, 2048)  # more lanes than the largest bucket
    with pytest.raises(Exception):
        R.build_rank_plan(g, 0, 64, port_base=65534)


def test_tp_pp_plans_agree():
    g = geometry(stages=(8, 8, 8, 8), gpus_per_node=8)
    plans = R.build_ring(g, 2, 32, quantization=R.Quantization.FP8_E4M3)
    assert len(plans) == 8
    for p in plans:
        assert p.tp_degree == 2 and p.rank == p.pp_stage_index * 2 + p.tp_rank
        assert p.tp_peer_ranks == [p.pp_stage_index * 2 + (1 - p.tp_rank)]
        assert p.tp_peer_ports == [R.DEFAULT_PORT_BASE + 100 + p.tp_peer_ranks[0]]
        assert p.quantization == R.Quantization.FP8_E4M3
        nc = TP.derive_node_config(TP.Shape(2, p.tp_rank, 4, p.pp_stage_index), g.tp_geometry, g.shape_inputs)
        assert p.shape_configuration_hash == nc.configuration_hash and p.first_layer == nc.first_layer_index
        if p.flags & R.FLAG_HAS_NEXT:
            assert p.next_rank == p.rank + 2 and plans[p.next_rank].previous_rank == p.rank
            assert p.output_endpoint.transport == "nvlink.peer_memory"  # one node of 8 GPUs
    # TP degree that does not divide the heads
    with pytest.raises(Exception):
        R.build_ring(g, 3, 32)
