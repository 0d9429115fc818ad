"""Tests that need two or more GPUs of one node (NCCL + NVLink peer memory).
Skipped when fewer GPUs are visible."""

import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs 2 GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@needs2
def test_peer_memory_zero_step_matches_single_process():
    import multi_gpu_workers as W
    mp.spawn(W.peer_dp_worker, args=(2, _port()), nprocs=2, join=True)


@needs2
def test_fused_tensor_parallel_matches_single_gpu():
    import multi_gpu_workers as W
    mp.spawn(W.tp_fused_worker, args=(2, _port()), nprocs=2, join=True)


@needs2
def test_fused_expert_parallel_matches_single_gpu():
    import multi_gpu_workers as W
    mp.spawn(W.ep_fused_worker, args=(2, _port()), nprocs=2, join=True)


@needs2
def test_context_parallel_kernels_match_single_gpu():
    import multi_gpu_workers as W
    mp.spawn(W.cp_kernel_worker, args=(2, _port()), nprocs=2, join=True)
