"""The all-gather fused into the GEMM epilogue (tk_gemm_f16_f16_f32_nn_gather) on
2, 4 and 8 GPUs, one process per GPU: every rank's gathered buffer holds every
rank's row block within the GEMM error bound of the FP64 oracle, its padding
untouched, and the ranks' copies are bit-identical. Each world size is skipped
when the machine has fewer GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, result_q):
    import datetime
    import hashlib
    import sys

    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path[:0] = [ROOT, os.path.join(ROOT, "thunderkittens-sm7x_b200")]
    import oracle
    import tk_b200
    from tk_b200 import dist as tkd

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    errors = []
    try:
        for m, n, k, ldc in shapes:
            # Rank r's rows of A and the shared B: seeded, N(0, 0.02^2), binary16 (the oracle's generator).
            blocks = []
            b_host = None
            for r in range(world):
                a_r, b_r = oracle.gen_gemm_normal(100 + r, 0.02, m, n, k, k, n)
                blocks.append(a_r)
                if b_host is None:
                    b_host = b_r
            to_dev = lambda x: torch.from_numpy(x.view(np.int16).copy()).view(torch.float16).cuda()  # noqa: E731
            a_dev, b_dev = to_dev(blocks[rank]), to_dev(b_host)
            buf = tkd.GatheredBuffer(world * m, ldc)
            view = buf.tensor()
            view.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            code = tk_b200.gemm_gather_raw(m, n, k, a_dev, k, b_dev, n, buf.ptrs, rank, ldc)
            torch.cuda.synchronize()
            dist.barrier()  # every rank's stores into this rank's buffer are done
            got = view.cpu().numpy()
            if code != 0:
                errors.append(f"rank {rank}: code {code} for {(m, n, k, ldc)}")
            digests = []
            for r in range(world):
                part = np.ascontiguousarray(got[r * m:(r + 1) * m])
                ref, sabs = oracle.gemm_ref(m, n, k, blocks[r], k, b_host, n)
                fails = oracle.gemm_check(k, part[:, :n], ref, sabs, n, n)[0]
                if fails:
                    errors.append(f"rank {rank}: block {r} of {(m, n, k, ldc)}: {fails} cells outside the bound")
                if ldc > n and not np.isnan(part[:, n:]).all():
                    errors.append(f"rank {rank}: padding of block {r} written for {(m, n, k, ldc)}")
                digests.append(hashlib.sha256(part[:, :n].tobytes()).hexdigest())
            everyone = [None] * world
            dist.all_gather_object(everyone, digests)
            if any(d != everyone[0] for d in everyone):
                errors.append(f"rank {rank}: the ranks' gathered copies differ for {(m, n, k, ldc)}")
            dist.barrier()
            buf.close()  # collective
        assert tk_b200.device_status() == 0
    except Exception as exc:  # reported to the parent
        errors.append(f"rank {rank}: {exc!r}")
    finally:
        dist.destroy_process_group()
    result_q.put((rank, errors))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_gather_fused(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    shapes = [(512, 1024, 2048, 1024), (256, 784, 512, 790), (1024, 2048, 1024, 2048)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    errors = [e for _, errs in results for e in errs]
    assert not errors, errors
