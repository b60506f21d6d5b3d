"""Tensor-parallel drafting on 2 GPUs (one process per GPU; LS_TP_TEST_WORLD
= 4 or 8 runs the same tests over more ranks): the fused row-parallel GEMM +
peer-store allreduce, the vocabulary-sharded Markov chain, and the whole round
against the oracle (fused and NCCL allreduce).  Skipped with fewer GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import tp_workers

pytestmark = pytest.mark.gpu

WORLD = int(os.environ.get("LS_TP_TEST_WORLD", "2"))


@pytest.fixture(autouse=True)
def _gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} CUDA devices")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, *args):
    mp.start_processes(fn, args=(WORLD, _port(), *args), nprocs=WORLD, join=True, start_method="spawn")


def test_tp_gemm_allreduce_matches_oracle():
    _run(tp_workers.gemm_worker)


def test_tp_markov_sharded_matches_one_gpu():
    _run(tp_workers.markov_worker)


@pytest.mark.parametrize("allreduce,wire", [("fused", "f32"), ("fused", "bf16"), ("nccl", "bf16")])
def test_tp_round_matches_oracle(allreduce, wire):
    _run(tp_workers.engine_worker, allreduce, wire)
