"""forge-runtime's sort + gather composition on a B200: the reference's
pipeline_sort_then_gather_100k (forge-runtime/tests/pipeline_tests.rs:172-210)
and GpuGather's u32 / u64 forms (forge-runtime/src/gather.rs:119-140), with
the results checked against the CPU oracle; plus the bounds check that the
reference kernel does not have."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture()
def ctx():
    from forge_runtime import ForgeContext
    c = ForgeContext.new()
    yield c
    c.close()


def test_pipeline_sort_then_gather_100k(ctx):
    from forge_runtime import GpuGather, Pipeline
    from forge_sort import GpuSorter
    sorter = GpuSorter.with_context(ctx.device(), ctx.queue())
    gather = GpuGather.with_context(ctx.device(), ctx.queue())
    n = 100_000
    data = orc.gen("u32", n, seed=7)
    buf = sorter.alloc_sort_buffer("u32", n)
    buf.copy_from_slice(data)
    idx = ctx.alloc_buffer(100 * 4)
    idx.view(np.uint32)[:] = np.arange(100, dtype=np.uint32)
    out = ctx.alloc_buffer(100 * 4)
    p = Pipeline.new(ctx)
    p.sort(sorter, buf)
    p.gather(gather, buf, idx, out, 100, False)
    p.execute()
    want = orc.sort_keys(data, "u32")
    assert np.array_equal(out.view(np.uint32), want[:100])
    assert np.array_equal(buf.as_slice(), want)
    buf.free()
    gather.close()
    sorter.close()


@pytest.mark.parametrize("n,count", [(1 << 20, 1 << 20), (1 << 20, 1000), (4097, 3)])
@pytest.mark.parametrize("wide", [False, True])
def test_gather_buffers_match_numpy(ctx, n, count, wide):
    """Context buffers (page-locked host memory): a whole permutation (the
    source is staged in HBM) and a few indices into a large source (read in
    place over the bus)."""
    from forge_runtime import GpuGather
    g = GpuGather.with_context(ctx.device(), ctx.queue())
    dt = np.uint64 if wide else np.uint32
    src_h = orc.gen("u64" if wide else "u32", n, seed=n)
    perm = np.random.default_rng(count).permutation(n)[:count].astype(np.uint32)
    src = ctx.alloc_buffer(n * src_h.itemsize)
    src.view(dt)[:] = src_h
    idx = ctx.alloc_buffer(count * 4)
    idx.view(np.uint32)[:] = perm
    out = ctx.alloc_buffer(count * src_h.itemsize)
    (g.gather_u64 if wide else g.gather_u32)(src, idx, out, count)
    assert np.array_equal(out.view(dt), src_h[perm])
    g.close()


def test_gather_device_tensors_with_source_len():
    import torch
    from forge_runtime import GpuGather
    g = GpuGather.new()
    src = torch.arange(1000, dtype=torch.int64, device="cuda") * 3
    idx = torch.tensor([999, 0, 500, 7], dtype=torch.int32, device="cuda")
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        g.gather_u64(src.data_ptr(), idx.data_ptr(), out.data_ptr(), 4)
    g.gather_u64(src.data_ptr(), idx.data_ptr(), out.data_ptr(), 4, source_len=1000)
    assert out.cpu().tolist() == [2997, 0, 1500, 21]
    g.close()


def test_pipeline_reports_out_of_range_index(ctx):
    from forge_runtime import GpuGather, Pipeline, PipelineError
    g = GpuGather.with_context(ctx.device(), ctx.queue())
    src = ctx.alloc_buffer(64 * 4)
    src.view(np.uint32)[:] = np.arange(64, dtype=np.uint32)
    idx = ctx.alloc_buffer(2 * 4)
    idx.view(np.uint32)[:] = [3, 64]
    out = ctx.alloc_buffer(2 * 4)
    p = Pipeline(ctx)
    p.gather(g, src, idx, out, 2, False)
    with pytest.raises(PipelineError.GpuExecution) as ei:
        p.execute()
    assert str(ei.value).startswith("GPU execution failed: ")
    # the context stays usable
    idx.view(np.uint32)[:] = [3, 63]
    p = Pipeline(ctx)
    p.gather(g, src, idx, out, 2, False)
    p.execute()
    assert out.view(np.uint32).tolist() == [3, 63]
    g.close()
