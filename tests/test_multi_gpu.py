"""Tests that need two or more GPUs of one node (NCCL + NVLink peer memory).
Each runs at 2, 4 and 8 ranks; a world larger than the number of visible
GPUs is skipped."""

import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLDS = [2, 4, 8]


def _need(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", WORLDS)
def test_peer_memory_zero_step_matches_single_process(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.peer_dp_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", WORLDS)
def test_peer_memory_step_under_model_parallel_layouts(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.peer_dp_layout_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", WORLDS)
def test_fully_sharded_matches_zero_step(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.fsdp_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", WORLDS)
def test_fused_tensor_parallel_matches_single_gpu(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.tp_fused_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", WORLDS)
def test_fused_expert_parallel_matches_single_gpu(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.ep_fused_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", WORLDS)
def test_context_parallel_kernels_match_single_gpu(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.cp_kernel_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_ring_context_parallel_matches_single_gpu(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.cp_kernel_worker, args=(world, _port(), "ring"), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_rank_leaving_between_steps_is_detected(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.rank_leave_worker, args=(world, _port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_pipeline_parallel_matches_single_gpu(world):
    _need(world)
    import multi_gpu_workers as W
    mp.spawn(W.pp_worker, args=(world, _port()), nprocs=world, join=True)
