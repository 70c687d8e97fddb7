"""The reference's known-answer tests, run through GpuSorter on the GPU
(transcribed in tests/golden/known_answers.json with file:line)."""
import numpy as np
import pytest

import _cases

pytestmark = pytest.mark.gpu
CASES = _cases.load()["cases"]


@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_known_answer(sorter, c):
    dt = c["dtype"]
    x = _cases.case_input(c)
    keys, idx, vals = _cases.expected(c)
    if c["op"] == "sort":
        a = x.copy()
        getattr(sorter, f"sort_{dt}")(a)
        assert _cases.as_bits(a, dt) == keys
        # the zero-copy buffer path gives the same answer
        buf = sorter.alloc_sort_buffer(dt, max(len(x), 1))
        buf.copy_from_slice(x)
        getattr(sorter, "sort_buffer" if dt == "u32" else f"sort_{dt}_buffer")(buf)
        assert _cases.as_bits(buf.as_slice(), dt) == keys
        buf.free()
    elif c["op"] == "argsort":
        before = x.copy()
        got = getattr(sorter, f"argsort_{dt}")(x)
        assert got.dtype == np.uint32
        assert [int(i) for i in got] == idx
        assert np.array_equal(x.view(np.uint8), before.view(np.uint8)), "argsort must not modify input"
    else:
        k, v = x.copy(), _cases.case_values(c).copy()
        getattr(sorter, f"sort_pairs_{dt}")(k, v)
        assert _cases.as_bits(k, dt) == keys
        assert [int(t) for t in v] == vals


def test_length_mismatch_fields(sorter):
    from forge_sort import LengthMismatch
    with pytest.raises(LengthMismatch) as ei:
        sorter.sort_pairs_u32(np.array([1, 2, 3], np.uint32), np.array([10, 20], np.uint32))
    assert (ei.value.keys, ei.value.values) == (3, 2)
    assert str(ei.value) == "length mismatch: keys=3, values=2"
    with pytest.raises(LengthMismatch):
        sorter.sort_pairs_i64(np.array([1, 2, 3], np.int64), np.array([10, 20], np.uint32))


@pytest.mark.parametrize("dt", ["u32", "i32", "f32", "u64", "i64", "f64"])
def test_empty_and_single(sorter, dt):
    npdt = _cases.NP[dt]
    e = np.empty(0, npdt)
    getattr(sorter, f"sort_{dt}")(e)
    assert e.size == 0
    one = np.array([42], npdt)
    getattr(sorter, f"sort_{dt}")(one)
    assert one[0] == 42
    assert getattr(sorter, f"argsort_{dt}")(e).size == 0
    assert list(getattr(sorter, f"argsort_{dt}")(one)) == [0]
    k, v = np.array([42], npdt), np.array([100], np.uint32)
    getattr(sorter, f"sort_pairs_{dt}")(k, v)
    assert k[0] == 42 and v[0] == 100
