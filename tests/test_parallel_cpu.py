"""Multi-rank CPU tests (Gloo): every parallel axis against the
single-process oracle; the workers live in ``dist_workers``."""

import socket

import pytest
import torch.multiprocessing as mp

import dist_workers as W  # noqa: E402


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, *args):
    mp.spawn(fn, args=(world, _port()) + args, nprocs=world, join=True)


@pytest.mark.parametrize("sp", [True, False])
@pytest.mark.parametrize("moe", [False, True])
def test_tensor_parallel_matches_single(sp, moe):
    _run(W.tp_worker, 2, sp, moe)


@pytest.mark.parametrize("mode", ["replicate", "shard"])
def test_data_parallel_matches_accumulation(mode):
    _run(W.dp_worker, 2, mode)


def test_expert_parallel_matches_single():
    _run(W.ep_worker, 2)


@pytest.mark.parametrize("moe", [False, True])
def test_context_parallel_matches_single(moe):
    _run(W.cp_worker, 2, moe)


@pytest.mark.parametrize("world,moe", [(2, False), (4, False), (2, True)])
def test_ring_context_parallel_matches_single(world, moe):
    """k|v blocks passed around the ring (two blocks per rank in memory)
    give the single-process loss, logits and every gradient."""
    _run(W.cp_worker, world, moe, "ring")


@pytest.mark.parametrize("tied,micro", [(False, 2), (True, 4)])
def test_pipeline_parallel_matches_accumulation(tied, micro):
    _run(W.pp_worker, 2, tied, micro)


def test_manager_grid_groups():
    _run(W.manager_worker, 4, 2, 1, 1, 2)


def test_heartbeat_detects_silent_rank():
    _run(W.heartbeat_worker, 3, 1)


def test_tensor_parallel_checkpoint_roundtrip_and_reshard(tmp_path):
    _run(W.tp_checkpoint_worker, 2, str(tmp_path))


def test_expert_parallel_checkpoint_loads_single_layout(tmp_path):
    _run(W.ep_checkpoint_worker, 2, str(tmp_path))


def test_global_batch_moe_balance():
    _run(W.global_balance_worker, 2)


def test_rank_leaving_between_steps_is_detected():
    _run(W.rank_leave_worker, 3)


def test_zero_shard_checkpoint_resumes_exactly(tmp_path):
    _run(W.zero_checkpoint_worker, 2, str(tmp_path))


def test_pipeline_parallel_checkpoint_loads_single_layout(tmp_path):
    _run(W.pp_checkpoint_worker, 2, str(tmp_path))


@pytest.mark.parametrize("moe,ckpt", [(False, False), (False, True), (True, False)])
def test_fully_sharded_matches_zero(moe, ckpt):
    _run(W.fsdp_worker, 2, moe, ckpt)


def test_fully_sharded_checkpoint_resumes_and_reshards(tmp_path):
    _run(W.fsdp_checkpoint_worker, 2, str(tmp_path))


def test_fully_sharded_reference_api_loop():
    _run(W.fsdp_api_worker, 2)


@pytest.mark.parametrize("world,ep", [(2, 2), (4, 2)])
def test_fully_sharded_with_expert_parallel(world, ep):
    _run(W.fsdp_ep_worker, world, ep)


@pytest.mark.parametrize("axis", ["tp_size", "cp_size"])
def test_sft_takes_model_parallel_layouts(tmp_path, axis):
    _run(W.sft_parallel_worker, 2, str(tmp_path), axis)


def test_peer_memory_groups_stay_on_one_node():
    """Groups that span nodes (torchrun's consecutive local ranks) are not
    given the peer-memory kernels."""
    from nano_qwen_b200.parallel.peer_dp import same_node
    assert same_node([0, 1, 2, 3], 8) and same_node([8, 9, 15], 8)
    assert not same_node([6, 7, 8, 9], 8)
    assert not same_node([0, 8], 8)       # an expert-data-parallel pair across nodes
    assert same_node([0, 8, 16], 0)       # size unknown: single-node launch


@pytest.mark.parametrize("world", [2, 4])
def test_peer_memory_zero_host_code_on_fake_transport(tmp_path, world):
    _run(W.peer_dp_fake_worker, world, str(tmp_path))


@pytest.mark.parametrize("world,tp,moe", [(4, 2, False), (2, 2, False), (4, 2, True)])
def test_fully_sharded_with_tensor_parallel(world, tp, moe):
    _run(W.fsdp_tp_worker, world, tp, moe)


def test_engine_under_pure_tensor_parallelism_matches_single():
    _run(W.tp_engine_worker, 2)


LAYOUTS = {
    "dp2": (2, {}),
    "tp2": (2, {"tp_size": 2}),
    "pp2": (2, {"pp_size": 2, "pp_microbatches": 2}),
    "cp2": (2, {"cp_size": 2}),
    "ep2-moe": (2, {"ep_size": 2, "moe": True}),
    "tp2xdp2": (4, {"tp_size": 2}),
    "pp2xdp2": (4, {"pp_size": 2, "pp_microbatches": 2}),
    "tp2xdp2-fsdp": (4, {"tp_size": 2, "shard_params": True}),
    "dp2-fsdp-moe": (2, {"moe": True, "shard_params": True}),
    "cp2xdp2": (4, {"cp_size": 2}),
    "cp2-ring": (2, {"cp_size": 2, "cp_mode": "ring"}),
    "ep2xdp2-moe": (4, {"ep_size": 2, "moe": True}),
    "ep2-fsdp-moe": (4, {"ep_size": 2, "moe": True, "shard_params": True}),
    "tp2xpp2": (4, {"tp_size": 2, "pp_size": 2, "pp_microbatches": 2}),
    "tp2xpp2-nosp": (4, {"tp_size": 2, "pp_size": 2, "pp_microbatches": 2, "sequence_parallel": False}),
    "tp2xcp2-nosp": (4, {"tp_size": 2, "cp_size": 2, "sequence_parallel": False}),
    "cp2-moe": (2, {"cp_size": 2, "moe": True}),
    "pp2-moe": (2, {"pp_size": 2, "pp_microbatches": 2, "moe": True}),
    "pp2xep2-moe": (4, {"pp_size": 2, "pp_microbatches": 2, "ep_size": 2, "moe": True}),
    "tp2-moe": (2, {"tp_size": 2, "moe": True}),
    "tp2xep2-moe": (4, {"tp_size": 2, "ep_size": 2, "moe": True, "sequence_parallel": False}),
    "dp2-accum2": (2, {"accum": 2}),
    "dp2-overlap": (2, {"overlap": True}),
    "dp2-overlap-accum2": (2, {"overlap": True, "accum": 2}),
    "tp2xdp2-overlap": (4, {"tp_size": 2, "overlap": True}),
    "dp2-overlap-tied": (2, {"overlap": True, "tied": True}),
    "tp2xdp2-fsdp-accum2": (4, {"tp_size": 2, "shard_params": True, "accum": 2}),
    "ep2-fsdp-moe-accum2": (2, {"ep_size": 2, "moe": True, "shard_params": True, "accum": 2}),
    "cp2xdp2-accum2": (4, {"cp_size": 2, "accum": 2}),
    "cp2-fsdp": (2, {"cp_size": 2, "shard_params": True}),
    "cp2xdp2-fsdp": (4, {"cp_size": 2, "shard_params": True}),
    "cp2-ring-fsdp-moe": (2, {"cp_size": 2, "cp_mode": "ring", "shard_params": True, "moe": True}),
    "pp2-fsdp": (2, {"pp_size": 2, "pp_microbatches": 2, "shard_params": True}),
    "pp2xdp2-fsdp": (4, {"pp_size": 2, "pp_microbatches": 2, "shard_params": True}),
    "pp2-tied": (2, {"pp_size": 2, "pp_microbatches": 2, "tied": True}),
    "pp2-fsdp-tied": (2, {"pp_size": 2, "pp_microbatches": 2, "shard_params": True, "tied": True}),
    "dp2-fsdp-tied": (2, {"shard_params": True, "tied": True}),
    "tp2-tied": (2, {"tp_size": 2, "tied": True}),
    "dp2-moe-balance": (2, {"moe": True, "balance": True}),
    "ep2-moe-balance": (2, {"ep_size": 2, "moe": True, "balance": True}),
    "dp2-fsdp-moe-balance": (2, {"moe": True, "balance": True, "shard_params": True}),
    "dp2-docs": (2, {"docs": True}),
    "tp2-docs": (2, {"tp_size": 2, "docs": True}),
    "pp2-docs": (2, {"pp_size": 2, "pp_microbatches": 2, "docs": True}),
    "tp2xpp2-docs": (4, {"tp_size": 2, "pp_size": 2, "pp_microbatches": 2, "docs": True}),
    "dp2-pad": (2, {"pad": True}),
    "tp2-pad": (2, {"tp_size": 2, "pad": True}),
    "pp2-pad": (2, {"pp_size": 2, "pp_microbatches": 2, "pad": True}),
    "ep2-moe-pad": (2, {"ep_size": 2, "moe": True, "pad": True}),
    "dp2-fsdp-pad-accum2": (2, {"shard_params": True, "pad": True, "accum": 2}),
    "tp2xdp2-pad": (4, {"tp_size": 2, "pad": True}),
    "cp2-pad": (2, {"cp_size": 2, "pad": True}),
}


@pytest.mark.parametrize("world", [2, 4])
def test_engine_layouts_match_single_process(world):
    """Every layout the manager builds trains like one process: the engine's
    loss and gradient norm over two steps (all layouts of one world size in
    one job; a failure names its layout)."""
    cases = [(n, lay) for n, (w, lay) in sorted(LAYOUTS.items()) if w == world]
    _run(W.layouts_worker, world, cases)


# the peer-memory data-parallel step (dp_mode="p2p") under model
# parallelism, its kernels restated over file-backed shared buffers
PEER_LAYOUTS = {
    "cp2-p2p": (2, {"cp_size": 2, "dp_mode": "p2p"}),
    "ep2-moe-p2p": (2, {"ep_size": 2, "moe": True, "dp_mode": "p2p"}),
    "dp2-moe-p2p": (2, {"moe": True, "dp_mode": "p2p"}),
    "tp2xdp2-p2p": (4, {"tp_size": 2, "dp_mode": "p2p"}),
    "pp2xdp2-p2p": (4, {"pp_size": 2, "pp_microbatches": 2, "dp_mode": "p2p"}),
    "cp2xdp2-p2p": (4, {"cp_size": 2, "dp_mode": "p2p"}),
    "ep2xdp2-moe-p2p": (4, {"ep_size": 2, "moe": True, "dp_mode": "p2p"}),
    "tp2xep2-moe-p2p": (4, {"tp_size": 2, "ep_size": 2, "moe": True, "sequence_parallel": False,
                            "dp_mode": "p2p"}),
    "pp2xep2-moe-p2p": (4, {"pp_size": 2, "pp_microbatches": 2, "ep_size": 2, "moe": True,
                            "dp_mode": "p2p"}),
    "ep2xdp2-moe-p2p-accum2": (4, {"ep_size": 2, "moe": True, "dp_mode": "p2p", "accum": 2}),
    "ep2-moe-balance-p2p": (2, {"ep_size": 2, "moe": True, "balance": True, "dp_mode": "p2p"}),
    "cp2-moe-p2p": (2, {"cp_size": 2, "moe": True, "dp_mode": "p2p"}),
    "tp2-moe-p2p-tied": (4, {"tp_size": 2, "moe": True, "tied": True, "dp_mode": "p2p"}),
    "tp2xdp2-p2p-config": (4, {"tp_size": 2, "dp_mode_cfg": "p2p"}),
    "tp2xdp2-default-nccl": (4, {"tp_size": 2, "expect_nccl": True}),
}


@pytest.mark.parametrize("world", [2, 4])
def test_peer_step_layouts_match_single_process(tmp_path, world):
    """The peer-memory step's host code (shard bounds, the expert span's own
    shard over the ranks holding the same experts, flag epochs, the norm
    over TP / PP) under each layout trains like one process."""
    cases = [(n, lay) for n, (w, lay) in sorted(PEER_LAYOUTS.items()) if w == world]
    _run(W.peer_layouts_worker, world, cases, str(tmp_path))


CKPT_LAYOUTS = ["dp2", "tp2", "pp2", "ep2-moe", "tp2xdp2-fsdp", "ep2-fsdp-moe", "tp2xpp2", "cp2",
                "cp2-fsdp", "ep2xdp2-moe-p2p", "tp2xdp2-p2p", "dp2-overlap"]


@pytest.mark.parametrize("world", [2, 4])
def test_layout_checkpoints_move_to_and_from_one_process(tmp_path, world):
    """A checkpoint of each layout resumes in one process, and one process's
    checkpoint resumes in each layout, both continuing with equal losses and
    gradient norms (all cases of one world size in one job)."""
    every = {**LAYOUTS, **PEER_LAYOUTS}
    cases = [(n, every[n][1], fs) for n in CKPT_LAYOUTS if every[n][0] == world
             for fs in (False, True)]
    _run(W.layout_ckpts_worker, world, cases, str(tmp_path))


@pytest.mark.parametrize("shard", [False, True])
def test_dpo_data_parallel_matches_single(shard):
    _run(W.dpo_layout_worker, 2, shard)
