"""m3_cuda_abs_max_static: ABS_MAX over a batch of device tensors with a
static scratch array instead of allocated memory.

Its results must equal, bit for bit, those of the existing ABS_MAX path (a
session running an ABS_MAX graph node) on the same data, on two calls in a
row: the second call shows that the first one left the static scratch ready
for reuse.  This file is named to be collected last so that it also runs
after every other GPU test in the same process.
"""

from __future__ import annotations

import numpy as np
import pytest


def _bits_f16(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint16)


def _bits_bf16(values: np.ndarray) -> np.ndarray:
    # any 16-bit pattern is a BF16 input; truncation keeps the value's range
    return (values.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _batch(m3, dtype: int, seed: int) -> list[np.ndarray]:
    """Raw storage arrays of `dtype`: ragged sizes, an empty tensor, one
    element, signed zeros, subnormals and an infinity."""
    rng = np.random.default_rng(seed)
    sizes = [1000, 4096 * 37 + 3, 0, 1, 1 << 20, 77]
    out = []
    for index, size in enumerate(sizes):
        values = rng.standard_normal(size).astype(np.float32) * np.float32(2.0 ** (index - 2))
        if size > 10:
            values[3] = -0.0
            values[5] = np.float32(1e-41) if dtype == m3.F32 else np.float32(3e-8)
        if index == 4:
            values[size // 2] = -np.inf
        if dtype == m3.F32:
            out.append(values)
        elif dtype == m3.F16:
            out.append(_bits_f16(np.clip(values, -60000, 60000)))
        else:
            out.append(_bits_bf16(values))
    return out


def _session_abs_max(m3, dtype: int, data: np.ndarray) -> tuple[int, int]:
    """(status, result bits) of the existing ABS_MAX path on `data`."""
    g = m3.Graph()
    x = g.value(m3.INPUT, dtype, (data.shape[0],))
    m = g.inferred("ABS_MAX", [x], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [x], [m])
    s = m3.Session(g)
    s.write(x, data)
    status, _ = s.run_status()
    result = s.read(m)
    if status != m3.OK:
        return status, None
    return status, int(result.view(np.uint32)[0])


def test_rejects_batches_beyond_the_static_limit(m3):
    """More tensors than the scratch holds fail before any device work (no
    GPU needed); an empty batch succeeds without touching a device."""
    n = m3.ABS_MAX_STATIC_MAX_TENSORS + 1
    with pytest.raises(m3.M3Failure) as failure:
        m3.abs_max_static(m3.F32, [16] * n, [4] * n, 16)
    assert failure.value.status == m3.INVALID_ARGUMENT
    assert str(m3.ABS_MAX_STATIC_MAX_TENSORS) in failure.value.message
    m3.abs_max_static(m3.F32, [], [], 16)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["F32", "F16", "BF16"])
def test_matches_session_abs_max_on_two_calls_in_a_row(m3, gpu, dtype_name):
    import torch

    dtype = getattr(m3, dtype_name)
    host = _batch(m3, dtype, seed=41 + dtype)
    expected = []
    for data in host:
        status, result = _session_abs_max(m3, dtype, data)
        assert status == m3.OK
        expected.append(result)

    device = torch.device("cuda", 0)
    storage = [torch.from_numpy(a.view(np.uint8).copy()).to(device) for a in host]
    # one input one element past a 16-byte boundary: the gather path
    shifted = torch.empty(host[0].nbytes + 16, dtype=torch.uint8, device=device)
    element = host[0].itemsize
    shifted[element:element + host[0].nbytes] = storage[0]
    pointers = [t.data_ptr() if t.numel() else 0 for t in storage]
    pointers.append(shifted.data_ptr() + element)
    counts = [a.shape[0] for a in host] + [host[0].shape[0]]
    expected.append(expected[0])

    maxima = torch.empty(len(pointers), dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    torch.cuda.synchronize(device)
    free_before = None
    for call in range(2):
        maxima.fill_(0x7FC0DEAD)
        torch.cuda.synchronize(device)
        if call == 1:
            free_before = torch.cuda.mem_get_info(device)[0]
        m3.abs_max_static(dtype, pointers, counts, maxima.data_ptr(), device=0, stream=stream)
        if call == 1:
            assert torch.cuda.mem_get_info(device)[0] == free_before
        got = [int(v) & 0xFFFFFFFF for v in maxima.cpu().tolist()]
        assert got == expected, f"call {call + 1}"


@pytest.mark.gpu
def test_nan_input_untouched_and_scratch_reusable(m3, gpu):
    import torch

    host = _batch(m3, m3.F32, seed=7)
    poisoned = [a.copy() for a in host]
    poisoned[1][12345] = np.nan
    expected = [_session_abs_max(m3, m3.F32, a) for a in poisoned]
    assert expected[1][0] == m3.OUT_OF_RANGE
    device = torch.device("cuda", 0)
    maxima = torch.empty(len(host), dtype=torch.int32, device=device)
    for data, failing in ((poisoned, 1), (host, None)):
        storage = [torch.from_numpy(a.copy()).to(device) for a in data]
        pointers = [t.data_ptr() if t.numel() else 0 for t in storage]
        counts = [a.shape[0] for a in data]
        maxima.fill_(0x7FC0DEAD)
        torch.cuda.synchronize(device)
        if failing is None:
            m3.abs_max_static(m3.F32, pointers, counts, maxima.data_ptr())
        else:
            with pytest.raises(m3.M3Failure) as failure:
                m3.abs_max_static(m3.F32, pointers, counts, maxima.data_ptr())
            assert failure.value.status == m3.OUT_OF_RANGE
            assert "input 1 " in failure.value.message
        got = [int(v) & 0xFFFFFFFF for v in maxima.cpu().tolist()]
        for index, value in enumerate(got):
            if index == failing:
                assert value == 0x7FC0DEAD  # left untouched
            else:
                reference = _session_abs_max(m3, m3.F32, data[index])
                assert reference[0] == m3.OK and value == reference[1]


@pytest.mark.gpu
def test_largest_batch_and_argument_errors(m3, gpu):
    import torch

    device = torch.device("cuda", 0)
    n = m3.ABS_MAX_STATIC_MAX_TENSORS
    rng = np.random.default_rng(3)
    host = [rng.standard_normal(100 + 13 * i).astype(np.float32) for i in range(n)]
    storage = [torch.from_numpy(a).to(device) for a in host]
    maxima = torch.zeros(n, dtype=torch.float32, device=device)
    for _ in range(2):
        m3.abs_max_static(m3.F32, [t.data_ptr() for t in storage], [a.shape[0] for a in host],
                          maxima.data_ptr())
        got = maxima.cpu().numpy()
        assert np.array_equal(got, np.array([np.abs(a).max() for a in host], dtype=np.float32))
    with pytest.raises(m3.M3Failure) as failure:
        m3.abs_max_static(m3.I32, [storage[0].data_ptr()], [4], maxima.data_ptr())
    assert failure.value.status == m3.INVALID_ARGUMENT
    with pytest.raises(m3.M3Failure) as failure:
        m3.abs_max_static(m3.F32, [storage[0].data_ptr()], [4], maxima.data_ptr() + 2)
    assert failure.value.status == m3.INVALID_ARGUMENT
    with pytest.raises(m3.M3Failure) as failure:
        m3.abs_max_static(m3.F32, [0], [4], maxima.data_ptr())
    assert failure.value.status == m3.INVALID_ARGUMENT
