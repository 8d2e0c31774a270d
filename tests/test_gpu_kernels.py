"""CUDA kernels vs the CPU oracle, through the C ABI (tensor wrappers in kvoff.ops).

FP8 payloads and scales must match bit for bit, NaN and Inf rows included;
restored bf16 values must match bit for bit (NaN results are written as 0xFFFF
by both). BF16 passthrough and store_kvcache are byte moves and must be
byte-exact over arbitrary bit patterns.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def to_bf16(bits: np.ndarray, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.uint8).numpy()


def special_pool(layers: int, num_blocks: int, block_size: int, heads: int, d: int,
                 seed: int = 0) -> np.ndarray:
    """Pool whose rows cycle through every codec branch plus random finite rows."""
    rows = workloads.special_rows(d, seed)
    shape = (2, layers, num_blocks, block_size, heads, d)
    total = int(np.prod(shape[:-1]))
    rng = np.random.default_rng([seed, 99])
    finite = workloads.f32_to_bf16_bits(rng.standard_normal((total, d), dtype=np.float32))
    finite[: total: 3] = np.resize(rows, (len(finite[: total: 3]), d))
    return finite.reshape(shape)


def empty_slots(n: int, g, device):
    payload = torch.empty((n, g.fp8_payload_bytes), dtype=torch.uint8, device=device)
    scale = torch.empty((n, g.fp8_scale_bytes), dtype=torch.uint8, device=device)
    return payload, scale


# Config-2 heads, config-4 per-rank shards (tp=8: 1 KV head; tp=2: 4), and odd
# head dims and block sizes that take the generic kernels.
@pytest.mark.parametrize("d,heads,block_size", [(128, 8, 256), (128, 1, 256), (128, 4, 256),
                                               (64, 4, 64), (256, 2, 32), (32, 3, 16),
                                               (4, 1, 256), (8, 2, 16), (80, 2, 16)])
def test_fp8_save_restore_bit_exact(cuda, d, heads, block_size):
    from kvoff import ops

    bits = special_pool(2, 5, block_size, heads, d)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    ids = [3, 0, 4]
    payload, scale = empty_slots(len(ids), g, cuda)
    ops.save_fp8(pool, ids, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    want_p, want_s = oracle.fp8_save_blocks(bits, ids)
    torch.cuda.synchronize()
    assert np.array_equal(u8(payload).reshape(want_p.shape), want_p)
    assert np.array_equal(u16(scale.view(torch.bfloat16)).reshape(want_s.shape), want_s)

    targets = [1, 2, 3]
    ops.restore_fp8(pool, targets, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    oracle.fp8_restore_blocks(bits, targets, want_p, want_s)
    torch.cuda.synchronize()
    assert np.array_equal(u16(pool), bits)


def test_kernels_match_the_reference_quantizer_run_on_the_gpu(cuda):
    """The reference's fp8_quantize / fp8_dequantize torch ops (kept verbatim in
    the drop-in module) run on the same CUDA tensors, as the reference engine
    runs them. Every row with finite values is bit-identical. Rows holding Inf
    or NaN follow the CPU reference's encodings in the kernels, and ATen's CUDA
    ops differ from those only in NaN sign bits, so NaN-ness is compared there."""
    from kvoff import ops
    from kvoff.cpu_prefix_cache import fp8_dequantize, fp8_quantize

    bits = special_pool(2, 4, 256, 8, 128, seed=5)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    ids, targets = [0, 2], [1, 3]
    payload, scale = empty_slots(2, g, cuda)
    ops.save_fp8(pool, ids, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    slot_shape = (2, pool.shape[1], *pool.shape[3:])
    scale_shape = (*slot_shape[:-1], 1)
    finite = ((bits & 0x7F80) != 0x7F80).all(-1)  # [2, L, NB, BS, H]
    for i, b in enumerate(ids):
        ref_p = torch.empty(slot_shape, dtype=torch.float8_e4m3fn, device=cuda)
        ref_s = torch.empty(scale_shape, dtype=torch.bfloat16, device=cuda)
        fp8_quantize(pool[:, :, b], ref_p, ref_s)
        ok = finite[:, :, b]
        got_p, want_p = u8(payload[i]).reshape(slot_shape), u8(ref_p)
        got_s, want_s = u16(scale[i].view(torch.bfloat16)).reshape(scale_shape), u16(ref_s)
        assert np.array_equal(got_p[ok], want_p[ok])
        assert np.array_equal(got_s[ok], want_s[ok])
        nan8 = lambda a: (a & 0x7F) == 0x7F  # noqa: E731
        assert np.array_equal(nan8(got_p[~ok]), nan8(want_p[~ok]))
        # Dequantize this slot with both and compare the finite rows.
        ref_out = torch.empty(slot_shape, dtype=torch.bfloat16, device=cuda)
        fp8_dequantize(payload[i].view(torch.float8_e4m3fn).view(slot_shape),
                       scale[i].view(torch.bfloat16).view(scale_shape), ref_out)
        ops.restore_fp8(pool, [targets[i]], [payload[i].data_ptr()], [scale[i].data_ptr()])
        got = u16(pool[:, :, targets[i]])
        assert np.array_equal(got[ok], u16(ref_out)[ok])


def test_fp8_restore_of_arbitrary_slot_bits(cuda):
    from kvoff import ops

    rng = np.random.default_rng(4)
    shape = (2, 2, 3, 64, 4, 128)
    bits = rng.integers(0, 1 << 16, shape).astype(np.uint16)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    p = rng.integers(0, 256, (2, g.fp8_payload_bytes)).astype(np.uint8)
    s = rng.integers(0, 1 << 16, (2, g.rows)).astype(np.uint16)
    dp, ds = torch.from_numpy(p).to(cuda), torch.from_numpy(s.view(np.int16)).to(cuda)
    ops.restore_fp8(pool, [2, 0], [x.data_ptr() for x in dp], [x.data_ptr() for x in ds])
    oracle.fp8_restore_blocks(bits, [2, 0], p.reshape(2, 2, 2, 64, 4, 128),
                              s.reshape(2, 2, 2, 64, 4, 1))
    torch.cuda.synchronize()
    assert np.array_equal(u16(pool), bits)


def test_fp8_config1_matches_reference_digests(cuda):
    """BASELINE config 1 at full size: 16 blocks of [2, 28, 256, 8, 128]."""
    from kvoff import ops

    golden = json.loads((GOLDEN / "config1.json").read_text())
    c = golden["config"]
    sources, targets = golden["sources"], golden["targets"]
    bits = workloads.pool_with_blocks(sources, c["layers"], c["num_blocks"], c["block_size"],
                                      c["heads"], c["head_dim"], c["seed"])
    pool = to_bf16(bits, cuda)
    del bits
    g = ops.geometry(pool)
    payload, scale = empty_slots(len(sources), g, cuda)
    ops.save_fp8(pool, sources, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    assert [sha(u8(p)) for p in payload] == golden["fp8"]["payload_sha256"]
    assert [sha(u8(s)) for s in scale] == golden["fp8"]["scale_sha256"]
    ops.restore_fp8(pool, targets, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    assert [sha(u16(pool[:, :, t])) for t in targets] == golden["fp8"]["restored_sha256"]


def test_fp8_staged_and_mapped_pinned_slots(cuda):
    from kvoff import ops
    from kvoff.slab import PinnedSlab

    bits = special_pool(3, 6, 256, 8, 128, seed=2)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    ids = [5, 1]
    n = len(ids)
    slab = PinnedSlab(2 * n * (g.fp8_payload_bytes + g.fp8_scale_bytes), device=0)
    half = n * (g.fp8_payload_bytes + g.fp8_scale_bytes)
    views = []
    for k in range(2):  # k=0 staged slots, k=1 mapped slots
        base = k * half
        payload = slab.view(base, (n, g.fp8_payload_bytes), torch.uint8)
        scale = slab.view(base + n * g.fp8_payload_bytes, (n, g.fp8_scale_bytes), torch.uint8)
        payload.fill_(0xAB)
        scale.fill_(0xCD)
        views.append((payload, scale))
    staging_p, staging_s = empty_slots(1, g, cuda)  # one block of staging: two rounds
    (hp, hs), (mp, ms) = views
    ops.save_fp8_staged(pool, ids, [p.data_ptr() for p in hp], [s.data_ptr() for s in hs],
                        staging_p, staging_s)
    ops.save_fp8(pool, ids, [slab.device_alias(p) for p in mp], [slab.device_alias(s) for s in ms],
                 max_ctas=64)
    torch.cuda.synchronize()
    want_p, want_s = oracle.fp8_save_blocks(bits, ids)
    for payload, scale in views:
        assert np.array_equal(payload.numpy().reshape(want_p.shape), want_p)
        assert np.array_equal(scale.numpy().view(np.uint16).reshape(want_s.shape), want_s)
    ops.restore_fp8_staged(pool, [0, 2], [p.data_ptr() for p in hp], [s.data_ptr() for s in hs],
                           staging_p, staging_s)
    ops.restore_fp8(pool, [3, 4], [slab.device_alias(p) for p in mp],
                    [slab.device_alias(s) for s in ms])
    oracle.fp8_restore_blocks(bits, [0, 2], want_p, want_s)
    oracle.fp8_restore_blocks(bits, [3, 4], want_p, want_s)
    torch.cuda.synchronize()
    assert np.array_equal(u16(pool), bits)


@pytest.mark.parametrize("serial", [False, True])
def test_fp8_staged_pipeline_over_many_groups_and_calls(cuda, serial):
    """Staging of 4 blocks runs as a two-half pipeline (kernels on a library
    stream); staging_blocks = 1 runs the same calls serially on the stream."""
    from kvoff import ops
    from kvoff.slab import PinnedSlab

    stream = torch.cuda.Stream(cuda)

    bits = special_pool(2, 12, 128, 8, 128, seed=6)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    per = g.fp8_payload_bytes + g.fp8_scale_bytes
    slab = PinnedSlab(7 * per, device=0)
    payload = [slab.view(i * g.fp8_payload_bytes, (g.fp8_payload_bytes,), torch.uint8)
               for i in range(7)]
    scale = [slab.view(7 * g.fp8_payload_bytes + i * g.fp8_scale_bytes, (g.fp8_scale_bytes,),
                       torch.uint8) for i in range(7)]
    staging = empty_slots(1 if serial else 4, g, cuda)
    ids = [11, 3, 7, 0, 5, 9, 1]
    want_p, want_s = oracle.fp8_save_blocks(bits, ids)
    for chunk in ([0, 1, 2, 3, 4], [5], [6]):  # one multi-group call, then two one-block calls
        ops.save_fp8_staged(pool, [ids[i] for i in chunk], [payload[i].data_ptr() for i in chunk],
                            [scale[i].data_ptr() for i in chunk], *staging, stream=stream)
    stream.synchronize()
    for i in range(7):
        assert np.array_equal(payload[i].numpy(), want_p[i].reshape(-1))
        assert np.array_equal(scale[i].numpy().view(np.uint16), want_s[i].reshape(-1))
    targets = [2, 4, 6, 8, 10, 11, 3]
    for chunk in ([0, 1, 2], [3, 4, 5, 6]):
        ops.restore_fp8_staged(pool, [targets[i] for i in chunk],
                               [payload[i].data_ptr() for i in chunk],
                               [scale[i].data_ptr() for i in chunk], *staging, stream=stream)
    oracle.fp8_restore_blocks(bits, targets, want_p, want_s)
    stream.synchronize()
    assert np.array_equal(u16(pool), bits)


def test_fp8_event_ordered_staged_calls(cuda):
    """The _ev entry points through the public wrappers: kernels ordered on
    given events, a source-read event, a restore done event, and a join."""
    from kvoff import ops
    from kvoff.slab import PinnedSlab

    bits = special_pool(2, 10, 128, 8, 128, seed=8)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    per = g.fp8_payload_bytes + g.fp8_scale_bytes
    slab = PinnedSlab(6 * per, device=0)
    payload = [slab.view(i * g.fp8_payload_bytes, (g.fp8_payload_bytes,), torch.uint8)
               for i in range(6)]
    scale = [slab.view(6 * g.fp8_payload_bytes + i * g.fp8_scale_bytes, (g.fp8_scale_bytes,),
                       torch.uint8) for i in range(6)]
    staging = empty_slots(2, g, cuda)
    stream = torch.cuda.Stream(cuda)
    ids = [9, 2, 5, 0, 7, 3]
    want_p, want_s = oracle.fp8_save_blocks(bits, ids)
    written = torch.cuda.Event()
    written.record(torch.cuda.current_stream(cuda))
    read = torch.cuda.Event()
    read.record(stream)
    for i in range(6):  # one block per call: kernels overlap the previous call's copies
        ops.save_fp8_staged(pool, [ids[i]], [payload[i].data_ptr()], [scale[i].data_ptr()],
                            *staging, stream=stream, wait_events=[written], source_done=read)
    torch.cuda.current_stream(cuda).wait_event(read)
    pool[:, :, ids[-1]].fill_(1.0)  # the last block is rewritten once it has been read
    stream.synchronize()
    for i in range(6):
        assert np.array_equal(payload[i].numpy(), want_p[i].reshape(-1))
        assert np.array_equal(scale[i].numpy().view(np.uint16), want_s[i].reshape(-1))
    targets = [1, 4, 6, 8, 9, 2]
    done = torch.cuda.Event()
    done.record(stream)
    for i in range(6):
        ops.restore_fp8_staged(pool, [targets[i]], [payload[i].data_ptr()],
                               [scale[i].data_ptr()], *staging, stream=stream, done_event=done)
    ops.join_pipeline(cuda, stream)
    stream.synchronize()
    oracle.fp8_restore_blocks(bits, targets, want_p, want_s)
    got = u16(pool)
    for t in targets:
        assert np.array_equal(got[:, :, t], bits[:, :, t])


def test_fp8_batches_larger_than_one_launch(cuda):
    from kvoff import ops

    bits = special_pool(1, 140, 16, 1, 128, seed=3)
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    ids = list(range(139, -1, -1))[:135]
    payload, scale = empty_slots(len(ids), g, cuda)
    ops.save_fp8(pool, ids, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    want_p, want_s = oracle.fp8_save_blocks(bits, ids)
    torch.cuda.synchronize()
    assert np.array_equal(u8(payload).reshape(want_p.shape), want_p)
    assert np.array_equal(u16(scale.view(torch.bfloat16)).reshape(want_s.shape), want_s)


@pytest.mark.parametrize("method", ["engine", "tma", "sm"])
@pytest.mark.parametrize("shape", [(2, 3, 6, 256, 8, 128), (2, 2, 4, 256, 1, 4)])
def test_bf16_passthrough_byte_exact(cuda, method, shape):
    from kvoff import ops
    from kvoff.slab import PinnedSlab

    code = {"engine": ops.COPY_ENGINE, "tma": ops.COPY_TMA, "sm": ops.COPY_SM}[method]
    rng = np.random.default_rng(len(shape) + shape[-1])
    bits = rng.integers(0, 1 << 16, shape).astype(np.uint16)  # NaN encodings included
    pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    nb = shape[2]
    ids, targets = [nb - 1, 1, 2], [0, nb - 2, nb - 1]
    if method == "tma":  # device slots only
        slots = torch.empty((len(ids), g.block_bytes), dtype=torch.uint8, device=cuda)
        ptrs = [s.data_ptr() for s in slots]
        host = None
    else:
        slab = PinnedSlab(len(ids) * g.block_bytes, device=0)
        host = slab.view(0, (len(ids), g.block_bytes), torch.uint8)
        ptrs = [slab.device_alias(s) if method == "sm" else s.data_ptr() for s in host]
    ops.copy_blocks(pool, ids, ptrs, method=code)
    torch.cuda.synchronize()
    got = (slots.cpu() if host is None else host).numpy()
    want = oracle.copy_blocks(bits, ids)
    assert np.array_equal(got.view(np.uint16).reshape(want.shape), want)
    ops.copy_blocks(pool, targets, ptrs, restore=True, method=code)
    oracle.copy_blocks(bits, targets, want, restore=True)
    torch.cuda.synchronize()
    assert np.array_equal(u16(pool), bits)
    from kvoff import device_error
    assert device_error(0) == 0


@pytest.mark.parametrize("staging_blocks", [1, 2, 3, 8])
@pytest.mark.parametrize("misaligned", [False, True])
def test_bf16_staged_copies_byte_exact(cuda, staging_blocks, misaligned):
    """kvoff_copy_blocks_staged: serial (one-block staging) and two-half
    pipelined staging, groups smaller than the batch, back-to-back calls on
    one ring, and a pool whose base is only 2-byte aligned (the SM-kernel
    fallback instead of TMA)."""
    from kvoff import device_error, ops
    from kvoff.slab import PinnedSlab

    shape = (2, 3, 9, 256, 2, 64)
    rng = np.random.default_rng(staging_blocks)
    bits = rng.integers(0, 1 << 16, shape).astype(np.uint16)
    if misaligned:  # same pool, one element into a larger buffer
        flat = torch.empty(int(np.prod(shape)) + 1, dtype=torch.bfloat16, device=cuda)
        pool = flat[1:].view(shape)
        pool.copy_(to_bf16(bits, cuda))
    else:
        pool = to_bf16(bits, cuda)
    g = ops.geometry(pool)
    ids, targets = [8, 0, 3, 5, 1], [2, 4, 6, 7, 0]
    slab = PinnedSlab(len(ids) * g.block_bytes, device=0)
    host = slab.view(0, (len(ids), g.block_bytes), torch.uint8)
    host.fill_(0xA5)
    staging = torch.empty((staging_blocks, g.block_bytes), dtype=torch.uint8, device=cuda)
    ptrs = [h.data_ptr() for h in host]
    ops.copy_blocks_staged(pool, ids[:2], ptrs[:2], staging)  # two calls share the ring
    ops.copy_blocks_staged(pool, ids[2:], ptrs[2:], staging)
    torch.cuda.synchronize()
    want = oracle.copy_blocks(bits, ids)
    assert np.array_equal(host.numpy().view(np.uint16).reshape(want.shape), want)
    ops.copy_blocks_staged(pool, targets, ptrs, staging, restore=True)
    oracle.copy_blocks(bits, targets, want, restore=True)
    ops.join_pipeline(cuda)
    torch.cuda.synchronize()
    assert np.array_equal(u16(pool), bits)
    assert device_error(0) == 0


def test_bounded_device_wait_reports_a_timeout_and_the_context_survives(cuda):
    """A device-side wait that nothing satisfies gives up after its limit and
    sets the flag the host reads; the context keeps working afterwards."""
    from kvoff import _lib, device_error, ops

    assert device_error(0) == 0
    stream = torch.cuda.current_stream(cuda)
    _lib.call("kvoff_debug_bounded_wait", 20_000_000, stream.cuda_stream)  # 20 ms
    assert device_error(0) & 1  # synchronizes, reads and clears
    assert device_error(0) == 0
    pool = torch.randint(-2 ** 15, 2 ** 15, (2, 2, 4, 16, 2, 64), dtype=torch.int16,
                         device=cuda).view(torch.bfloat16)
    g = ops.geometry(pool)
    slot = torch.empty(g.block_bytes, dtype=torch.uint8, device=cuda)
    ops.copy_blocks(pool, [3], [slot.data_ptr()], method=ops.COPY_TMA)
    assert torch.equal(slot.view(torch.int16), pool[:, :, 3].contiguous().view(torch.int16).reshape(-1))
    assert device_error(0) == 0


@pytest.mark.parametrize("name", sorted(workloads.STORE_CASES))
def test_store_kvcache_matches_oracle_and_fixture(cuda, name):
    from kvoff import ops

    golden = json.loads((GOLDEN / "store_kvcache.json").read_text())[name]
    n, h, d, nb, bs, pad = workloads.STORE_CASES[name]
    qkv, slots, k_in, v_in = workloads.store_kvcache_inputs(name)
    rows = to_bf16(qkv, cuda)
    key = rows[:, pad:pad + h * d].view(n, h, d)
    value = rows[:, pad + h * d:].view(n, h, d)
    k_cache, v_cache = to_bf16(k_in, cuda), to_bf16(v_in, cuda)
    slot_mapping = torch.from_numpy(slots).to(cuda)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.store_kvcache(key, value, k_cache, v_cache, slot_mapping, bad_slots=bad)
    assert sha(u16(k_cache)) == golden["k_cache_sha256"]
    assert sha(u16(v_cache)) == golden["v_cache_sha256"]
    assert int(bad.item()) == 0


def test_store_kvcache_graph_capture_and_bad_slots(cuda):
    from kvoff import ops

    n, h, d, nb, bs = 64, 8, 128, 4, 32
    torch.manual_seed(0)
    key = torch.randn(n, h, d, dtype=torch.bfloat16, device=cuda)
    value = torch.randn(n, h, d, dtype=torch.bfloat16, device=cuda)
    k_cache = torch.zeros(nb, bs, h, d, dtype=torch.bfloat16, device=cuda)
    v_cache = torch.zeros_like(k_cache)
    slots = torch.full((n,), -1, dtype=torch.int32, device=cuda)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.Stream(cuda)
    stream.wait_stream(torch.cuda.current_stream(cuda))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        ops.store_kvcache(key, value, k_cache, v_cache, slots, bad_slots=bad)  # warm up
        with torch.cuda.graph(graph, stream=stream):
            ops.store_kvcache(key, value, k_cache, v_cache, slots, bad_slots=bad)
    torch.cuda.current_stream(cuda).wait_stream(stream)
    mapping = torch.randperm(nb * bs, device=cuda)[:n].to(torch.int32)
    mapping[::5] = -1
    mapping[7] = nb * bs + 3  # out of range: skipped and counted
    slots.copy_(mapping)
    graph.replay()
    torch.cuda.synchronize()
    valid = (mapping >= 0) & (mapping < nb * bs)
    idx = mapping[valid].long()
    assert torch.equal(k_cache.view(-1, h * d)[idx], key.reshape(n, -1)[valid])
    assert torch.equal(v_cache.view(-1, h * d)[idx], value.reshape(n, -1)[valid])
    untouched = torch.ones(nb * bs, dtype=torch.bool, device=cuda)
    untouched[idx] = False
    assert not k_cache.view(-1, h * d)[untouched].any()
    assert int(bad.item()) == 1


def _reference_store_kvcache():
    """The reference's own store_kvcache (nanovllm/layers/attention.py:10-40, its
    Triton kernel and launcher) from the installed copy under baseline/_ref,
    loaded by path without the package's model imports; None when absent."""
    import importlib.util
    import sys
    import types

    tree = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "nanovllm_upstream" / "nanovllm"
    if not (tree / "layers" / "attention.py").exists():
        return None
    for package, path in (("nanovllm", tree), ("nanovllm.utils", tree / "utils"),
                          ("nanovllm.layers", tree / "layers")):
        if package not in sys.modules:
            module = types.ModuleType(package)
            module.__path__ = [str(path)]
            sys.modules[package] = module
    for name, rel in (("nanovllm.utils.context", "utils/context.py"),
                      ("nanovllm.layers.attention", "layers/attention.py")):
        if name not in sys.modules:
            spec = importlib.util.spec_from_file_location(name, tree / rel)
            module = importlib.util.module_from_spec(spec)
            sys.modules[name] = module
            spec.loader.exec_module(module)
    return sys.modules["nanovllm.layers.attention"].store_kvcache


@pytest.mark.parametrize("name", sorted(workloads.STORE_CASES))
def test_store_kvcache_matches_the_reference_triton_kernel_on_the_gpu(cuda, name):
    """kvoff's store and the reference's own Triton store_kvcache_kernel, both
    run on this GPU over the same arbitrary bit patterns, leave byte-identical
    caches (the Triton kernel moves bf16 loads and stores unchanged)."""
    from kvoff import ops

    ref_store = _reference_store_kvcache()
    if ref_store is None:
        pytest.skip("the reference's installed copy (baseline/_ref) is absent")
    n, h, d, nb, bs, pad = workloads.STORE_CASES[name]
    qkv, slots, k_in, v_in = workloads.store_kvcache_inputs(name)
    rows = to_bf16(qkv, cuda)
    key = rows[:, pad:pad + h * d].view(n, h, d)
    value = rows[:, pad + h * d:].view(n, h, d)
    slot_mapping = torch.from_numpy(slots).to(cuda)
    caches = {}
    for arm in ("kvoff", "reference"):
        k_cache, v_cache = to_bf16(k_in, cuda), to_bf16(v_in, cuda)
        store = ops.store_kvcache if arm == "kvoff" else ref_store
        store(key, value, k_cache, v_cache, slot_mapping)
        caches[arm] = (u16(k_cache), u16(v_cache))
    assert np.array_equal(caches["kvoff"][0], caches["reference"][0])
    assert np.array_equal(caches["kvoff"][1], caches["reference"][1])


@pytest.mark.parametrize("heads,dim,offset", [(2, 128, 0), (4, 128, 0), (8, 256, 0), (8, 128, 4),
                                              (3, 80, 0)])
def test_store_kvcache_row_shapes(cuda, heads, dim, offset):
    """Rows of 512 B, 1 KB (the row kernel at 32 / 64 threads per token), 4 KB
    (the general kernel, two vectors per thread), a source 8-byte aligned only
    (the general kernel at 8-byte vectors) and a 480-byte row: every valid token
    lands byte for byte, skipped and out-of-range slots leave the cache as it was."""
    from kvoff import ops

    n, nb, bs = 200, 6, 64
    row = heads * dim
    torch.manual_seed(heads * 1000 + dim + offset)
    raw = torch.randn(n * (2 * row + 8) + 8, device=cuda).to(torch.bfloat16)
    qkv = raw[offset:offset + n * (2 * row + 8)].view(n, 2 * row + 8)
    key = qkv[:, 8:8 + row].view(n, heads, dim)
    value = qkv[:, 8 + row:].view(n, heads, dim)
    k_cache = torch.randn(nb, bs, heads, dim, device=cuda).to(torch.bfloat16)
    v_cache = torch.randn_like(k_cache)
    k_want, v_want = k_cache.clone(), v_cache.clone()
    slots = torch.randperm(nb * bs, device=cuda)[:n].to(torch.int32)
    slots[::7] = -1
    slots[5] = nb * bs + 1
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.store_kvcache(key, value, k_cache, v_cache, slots, bad_slots=bad)
    valid = (slots >= 0) & (slots < nb * bs)
    idx = slots[valid].long()
    k_want.view(-1, row)[idx] = key.reshape(n, -1)[valid]
    v_want.view(-1, row)[idx] = value.reshape(n, -1)[valid]
    torch.cuda.synchronize()
    assert torch.equal(k_cache.view(torch.int16), k_want.view(torch.int16))
    assert torch.equal(v_cache.view(torch.int16), v_want.view(torch.int16))
    assert int(bad.item()) == 1
