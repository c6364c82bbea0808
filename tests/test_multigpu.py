"""Context parallelism across real GPUs: one process per GPU, CUDA-IPC peer memory, NCCL + gloo.

The CP run and a single-GPU run of the same bf16 weights are both compared with a float32 oracle
of the model (models/reference_model.py): the CP error must stay at the single-GPU error level
(both are bf16 pipelines; they differ only in reduction order), and the greedy tokens must agree.
Skipped when fewer than two GPUs are visible.
"""

import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

STEPS = 6


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from hetero_cp_ringattn_b200.config import preset
    cfg = preset("llama-3.2-1b")
    cfg.num_layers = 3
    return cfg


def _run(eng, prompt, chunks, strategy):
    tok, logits = eng.prefill(1, prompt, chunks, strategy, decode_horizon=STEPS + 1,
                              return_logits=True)
    toks = [int(tok)]
    cur = tok
    for _ in range(STEPS):
        cur = eng.decode_step([1], cur)
        toks.append(int(cur))
    eng.release(1)
    return toks, logits.float().cpu()


def _worker(rank, world, port, chunks, strategy, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from hetero_cp_ringattn_b200.models import reference_model
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=120))
    group = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    try:
        cfg = _cfg()
        hf = ModelWeights.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16)
        w = PreparedWeights.from_weights(hf)
        L = sum(chunks)
        prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(5))
        eng = LlamaCPEngine(cfg, w, rank=rank, world=world, device=dev, group=group,
                            max_context=L, max_batch=1, decode_reserve=16)
        res = _run(eng, prompt, chunks, strategy)
        eng.check_device()
        eng.close()
        if rank == 0:
            single = LlamaCPEngine(cfg, w, device=dev, max_context=L, max_batch=1, decode_reserve=16)
            ref = _run(single, prompt, [L], "vanilla")
            single.close()
            oracle = reference_model.forward(hf, prompt.to(dev), last_only=True)[0].float().cpu()
            torch.save({"cp": res, "single": ref, "oracle": oracle}, out)
        dist.barrier(group=group)
    finally:
        dist.destroy_process_group()


def _launch(chunks, strategy):
    world = len(chunks)
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "r.pt")
        mp.start_processes(_worker, args=(world, free_port(), chunks, strategy, out), nprocs=world,
                           join=True, start_method="spawn")
        return torch.load(out)


def _check(r):
    cp_toks, cp_logits = r["cp"]
    one_toks, one_logits = r["single"]
    oracle = r["oracle"]
    err_cp = (cp_logits - oracle).abs()
    err_one = (one_logits - oracle).abs()
    # the CP pipeline is as accurate as the single-GPU pipeline against the fp32 oracle
    assert err_cp.mean() <= 1.25 * err_one.mean() + 1e-3
    assert err_cp.max() <= 0.15 and err_one.max() <= 0.15
    assert (cp_logits - one_logits).abs().mean() < 1e-2
    assert int(torch.argmax(cp_logits)) == int(torch.argmax(oracle))
    assert cp_toks == one_toks


@pytest.mark.parametrize("chunks,strategy", [([1536, 1536], "vanilla"), ([2048, 1024], "zigzag"),
                                             ([1000, 1100], "striped")])
def test_two_gpu_cp_matches_single_gpu(chunks, strategy):
    _check(_launch(chunks, strategy))


@pytest.mark.parametrize("chunks,strategy", [
    ([1280, 1280, 256], "zigzag"),                                   # capacity ratio 5:5:1
    ([768, 768, 768, 768], "striped"),
    ([640, 640, 640, 640, 256, 256, 128, 128], "zigzag"),            # 5:5:5:5:2:2:1:1
    ([500, 400, 300, 200, 600, 700, 100, 300], "vanilla"),
])
def test_many_gpu_uneven_cp_matches_single_gpu(chunks, strategy):
    """3, 4 and 8 ranks with the capacity-weighted uneven splits (skipped below that many GPUs)."""
    _check(_launch(chunks, strategy))
