"""world_size-2 gloo tests of the multi-GPU host logic on CPU: column sharding + all-gather, data-parallel
batch split, and a rank failure seen by its peer as an error (never as a hang).

The local linear is a float stand-in (the sharding and gather logic is what is under test here); the CUDA
path of the same classes is exercised on the GPU in test_gpu_dist.py.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    try:
        q.put((rank, "ok", fn(rank, world)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, "err", f"{type(exc).__name__}: {exc}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def run_ranks(fn, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, st, val = q.get(timeout=timeout)
        out[rank] = (st, val)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def _column_parallel(rank, world):
    from comfy_quant_bench_b200.dist import ColumnParallelLinear, shard_bounds
    g = torch.Generator().manual_seed(0)
    w = torch.randn(12, 8, generator=g)
    x = torch.randn(5, 8, generator=g)
    a, b = shard_bounds(12, rank, world)
    lin = ColumnParallelLinear(lambda x2: x2 @ w[a:b].t(), 12, rank, world)
    y = lin(x)
    return float((y - x @ w.t()).abs().max())


def _affine_shards(rank, world):
    from comfy_quant_bench_b200.dist import shard_affine
    q = torch.arange(8 * 4, dtype=torch.int8).reshape(8, 4)
    s = torch.arange(2 * 8, dtype=torch.float32).reshape(2, 8)
    qs, ss, zs, bs = shard_affine(q, s, s + 100, torch.arange(8.0), rank, world)
    lo = rank * 4
    assert torch.equal(qs, q[lo:lo + 4]) and torch.equal(ss, s[:, lo:lo + 4]) and torch.equal(bs, torch.arange(8.0)[lo:lo + 4])
    return tuple(qs.shape)


def _split(rank, world):
    from comfy_quant_bench_b200.dist import split_batch
    x = torch.arange(5)
    return split_batch(x, rank, world).tolist()


def _one_rank_fails(rank, world):
    if rank == 1:
        raise RuntimeError("rank 1 dies before the collective")
    t = torch.zeros(2)
    dist.all_reduce(t)   # the peer never joins: gloo's timeout turns this into an error
    return "unreachable"


def test_column_parallel_gather_equals_full_matmul():
    out = run_ranks(_column_parallel)
    assert all(st == "ok" and val < 1e-5 for st, val in out.values()), out


def test_affine_shards_slice_rows_and_scale_columns():
    out = run_ranks(_affine_shards)
    assert out[0] == ("ok", (4, 4)) and out[1] == ("ok", (4, 4))


def test_split_batch_covers_the_batch_once():
    out = run_ranks(_split)
    assert out[0][1] + out[1][1] == [0, 1, 2, 3, 4]


def test_a_failed_rank_surfaces_as_an_error_on_its_peer():
    out = run_ranks(_one_rank_fails, timeout=90)
    assert out[1][0] == "err"
    assert out[0][0] == "err"       # the survivor gets an error from its collective, not a hang


def test_shard_bounds_reject_uneven_split():
    from comfy_quant_bench_b200.dist import shard_bounds
    with pytest.raises(ValueError):
        shard_bounds(10, 0, 4)


def test_head_parallel_rows_partition_the_fused_weight():
    """The head-parallel shards of a fused [parts * hidden, K] weight (q | k | v) cover every row exactly once, and
    each rank's rows come out part by part, heads in order (the local output layout [S, parts, H/P, D])."""
    from comfy_quant_bench_b200.ltx import _head_rows
    hidden, heads, world = 512, 8, 4
    d, hp = hidden // heads, heads // world
    for parts in (1, 2, 3):
        shards = [_head_rows(hidden, parts, r * hp, (r + 1) * hp, d) for r in range(world)]
        rows = sorted(x for sh in shards for x in sh)
        assert rows == list(range(parts * hidden))
        for r, sh in enumerate(shards):
            for p in range(parts):
                block = sh[p * hp * d:(p + 1) * hp * d]
                assert block == list(range(p * hidden + r * hp * d, p * hidden + (r + 1) * hp * d))


def _oracle_ops():
    """CPU stand-ins for the three library calls RowParallelW4A8 makes, built on the oracle (test only): the rotated
    slice's NaN-ignoring maxima and NaN flags, quantization with a given maximum, and the affine GEMM."""
    import types
    import numpy as np
    from oracle import ref

    def _rotated(x2, rot):
        bits = x2.contiguous().view(torch.int16).numpy().view(np.uint16)
        return ref.fwht_stages(ref.bf16_bits_to_f32(bits), rot)

    def rotquant_absmax(x2, rot, m_pad=None):
        v = _rotated(x2, rot)
        mp = m_pad or v.shape[0]
        out = np.zeros((2, mp), np.float32)
        out[0, :v.shape[0]] = np.nan_to_num(np.abs(v), nan=0.0).max(axis=1)
        out[1, :v.shape[0]] = np.isnan(v).any(axis=1)
        return torch.from_numpy(out)

    def rotquant_scaled(x2, rot, amax, m_pad=None, group_sums=False, kperm=False):
        v = _rotated(x2, rot)
        m = v.shape[0]
        scale = np.maximum(amax[0, :m].numpy() * np.float32(1.0 / 127.0), np.float32(1e-10)).astype(np.float32)
        inv = (np.float32(1.0) / scale).astype(np.float32)
        q = np.clip(np.rint(v * inv[:, None]), -127, 127).astype(np.int16)
        return torch.from_numpy(q), torch.from_numpy(scale), None

    def gemm_affine(a, sa, gs, qweight, scale, zeros, bias, a_kperm=False, zeros_prepared=None):
        y = ref.linear_affine(a.numpy(), sa.numpy(), ref.unpack_uint4(qweight.numpy()), scale.numpy(),
                              zeros_prepared.numpy(), None if bias is None else bias.numpy())
        return torch.from_numpy(y.astype(np.float32))

    return types.SimpleNamespace(rotquant_absmax=rotquant_absmax, rotquant_scaled=rotquant_scaled,
                                 gemm_affine=gemm_affine, prepare_affine_zeros=lambda z, g: z,
                                 rotquant=None)


def _row_parallel(rank, world):
    import sys
    import numpy as np
    from comfy_quant_bench_b200 import dist as cqdist
    from oracle import ref
    stand_in = _oracle_ops()
    sys.modules["comfy_quant_bench_b200.ops"] = stand_in          # the protocol under test, on CPU kernels
    import comfy_quant_bench_b200
    comfy_quant_bench_b200.ops = stand_in
    m, n, k, rot = 6, 16, 1024, 256
    x_bits = ref.synth_activations(m, k, seed=3)
    w = ref.synth_weight(n, k, seed=4)
    qw_u4, s, z = ref.weight_quant_affine(w, rot, 128)
    bias = ref.synth_bias(n, seed=5).astype(np.float32)
    packed = torch.from_numpy(ref.pack_int4(qw_u4.astype(np.int16)).view(np.uint8).view(np.int8))
    layer = cqdist.RowParallelW4A8(packed, torch.from_numpy(s), torch.from_numpy(z), torch.from_numpy(bias), rank,
                                   world, convrot_groupsize=rot)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
    kl = k // world
    y = layer(x[:, rank * kl:(rank + 1) * kl]).numpy().astype(np.float64)
    qx, sx = ref.rotquant(x_bits, rot, "int8")
    want = ref.linear_affine(qx, sx, qw_u4, s, z, bias)
    return float(np.abs(y - want).max() / np.abs(want).max())


def test_row_parallel_protocol_matches_the_full_linear():
    """RowParallelW4A8 over 2 gloo ranks with oracle stand-ins for the kernels: the combined per-token maxima give
    the full row's codes and scales, and the summed partials (bias once) equal the full linear to fp32 rounding."""
    out = run_ranks(_row_parallel)
    for rank in range(2):
        st, val = out[rank]
        assert st == "ok", val
        assert val <= 1e-5, val
