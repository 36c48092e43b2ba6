"""Fused launches in the backend plug-in (m3_cuda_backend_execute).

The reference's scheduler hands a backend whole command lists
(src/m3_graph_session.c:116-150, src/m3_backend.c:113-154).  The plug-in
merges consecutive element-wise commands over one output shape, and
SOFTMAX / TOP_K / ROW_SUM commands over one input view, into one launch.
These tests check that merging never changes a result: every output equals
what the reference's command-by-command order produces (F32 statements for
ADD / MUL / COPY, which are bit-exact; the unfused plug-in for the row
operators), including lists whose views alias, overlap in part or broadcast,
and that a failing data check still leaves the failing command's outputs and
everything after it untouched."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


class Plugin:
    """A plug-in context with host-side storage bookkeeping (the reference's
    backend layer holds it), F32 storages and arbitrary views."""

    def __init__(self, m3):
        self.m3 = m3
        self.lib = m3.load()
        self.storages = {}
        self.sizes = {}
        self.err = m3.M3Error()

        @m3.STORAGE_DATA
        def storage_data(storage):
            return self.storages[storage]

        self._keep = storage_data
        options = m3.BackendOptions(0, storage_data, False)
        self.context = ctypes.c_void_p()
        m3.check(self.lib.m3_cuda_backend_context_create(
            ctypes.byref(options), ctypes.byref(self.context), ctypes.byref(self.err)), self.err)

    def tensor(self, array):
        array = np.ascontiguousarray(array)
        handle, data = ctypes.c_void_p(), ctypes.c_void_p()
        self.m3.check(self.lib.m3_cuda_backend_allocate(
            self.context, max(array.nbytes, 4), 256, ctypes.byref(handle), ctypes.byref(data),
            ctypes.byref(self.err)), self.err)
        key = len(self.storages) + 1
        self.storages[key] = data.value
        self.sizes[key] = array.nbytes
        self.write(key, array)
        return key

    def write(self, key, array):
        array = np.ascontiguousarray(array)
        self.m3.check(self.lib.m3_cuda_backend_write(
            self.context, self.storages[key], 0, array.ctypes.data, array.nbytes,
            ctypes.byref(self.err)), self.err)

    def read(self, key, dtype=np.float32):
        host = np.zeros(self.sizes[key] // np.dtype(dtype).itemsize, dtype)
        self.m3.check(self.lib.m3_cuda_backend_read(
            self.context, self.storages[key], 0, host.ctypes.data, host.nbytes,
            ctypes.byref(self.err)), self.err)
        return host

    def view(self, key, shape, offset=0, strides=None, dtype=None, item=4):
        """A view of `shape` at element `offset`; `strides` in elements
        (default: row-major contiguous)."""
        v = self.m3.TensorView()
        v.metadata.dtype = self.m3.F32 if dtype is None else dtype
        v.metadata.rank = len(shape)
        if strides is None:
            strides, step = [], 1
            for n in reversed(shape):
                strides.insert(0, step)
                step *= n
        for i, n in enumerate(shape):
            v.metadata.shape[i] = n
            v.byte_strides[i] = strides[i] * item
        count = int(np.prod(shape))
        v.metadata.element_count = count
        v.metadata.byte_count = count * item
        v.byte_offset = offset * item
        v.storage = key
        return v

    def execute(self, commands):
        """commands: (kind, fields) with fields a dict of descriptor members."""
        cmd = (self.m3.Command * len(commands))()
        keep = []
        for i, (kind, member, fields) in enumerate(commands):
            cmd[i].kind = self.m3.OPS[kind]
            desc = getattr(cmd[i].descriptor, member)
            for name, value in fields.items():
                if isinstance(value, int):
                    setattr(desc, name, value)
                else:
                    keep.append(value)
                    setattr(desc, name, ctypes.pointer(value))
        status = self.lib.m3_cuda_backend_execute(self.context, cmd, len(commands), None,
                                                  ctypes.byref(self.err))
        return status, self.err.message.decode() if status != self.m3.OK else ""

    def launches(self):
        return self.lib.m3_cuda_backend_launch_count(self.context)

    def close(self):
        for key in list(self.storages):
            self.lib.m3_cuda_backend_free_storage(self.context, self.storages[key],
                                                  self.storages[key])
        self.lib.m3_cuda_backend_destroy_context(self.context)


def binary(kind, left, right, out):
    return (kind, "add", {"left": left, "right": right, "output": out})


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture
def plugin(m3, gpu):
    p = Plugin(m3)
    yield p
    p.close()


def test_c1_chain_is_one_launch(m3, plugin):
    """y = (x * c) + b as the reference issues it (MUL into a temporary, ADD
    from it), c and b broadcast over rows: one launch, both outputs written,
    bit-exact with the F32 statements."""
    rng = np.random.default_rng(5)
    rows, width = 64, 4096
    x = rng.uniform(-1, 1, (rows, width)).astype(np.float32)
    c = rng.uniform(0.5, 2, width).astype(np.float32)
    b = rng.standard_normal(width).astype(np.float32)
    kx, kc, kb = plugin.tensor(x), plugin.tensor(c), plugin.tensor(b)
    kt, ky = plugin.tensor(np.zeros_like(x)), plugin.tensor(np.zeros_like(x))
    status, message = plugin.execute([
        binary("MUL", plugin.view(kx, (rows, width)), plugin.view(kc, (width,)),
               plugin.view(kt, (rows, width))),
        binary("ADD", plugin.view(kt, (rows, width)), plugin.view(kb, (1, width)),
               plugin.view(ky, (rows, width))),
    ])
    assert status == m3.OK, message
    assert plugin.launches() == 1
    t = x * c
    assert np.array_equal(bits(plugin.read(kt)), bits(t.ravel()))
    assert np.array_equal(bits(plugin.read(ky)), bits((t + b).ravel()))


def _emulate(buffers, commands):
    """The reference's order: each command reads memory, then writes it."""
    import numpy.lib.stride_tricks as st

    for kind, (lk, lshape, loff, lstr), (rk, rshape, roff, rstr), (ok, oshape, ooff) in commands:
        def read(key, shape, off, strides):
            base = buffers[key]
            itemsz = base.itemsize
            v = st.as_strided(base[off:], shape=shape, strides=[s * itemsz for s in strides])
            return np.broadcast_to(v.copy(), oshape)

        a = read(lk, lshape, loff, lstr)
        if kind == "COPY":
            result = a.copy()
        else:
            b = read(rk, rshape, roff, rstr)
            result = a + b if kind == "ADD" else a * b
        count = int(np.prod(oshape))
        buffers[ok][ooff:ooff + count] = result.astype(np.float32).ravel()


def test_random_aliasing_lists_match_command_order(m3, plugin):
    """Random lists of ADD / MUL / COPY over three buffers whose views are
    windows at row offsets (exact aliases, partial overlaps), row or scalar
    broadcasts: every buffer equals the command-by-command result bit for
    bit, whatever the plug-in merged."""
    rng = np.random.default_rng(11)
    rows, width, nbuf = 6, 32, 3
    span = rows * width
    size = span + 3 * width
    checked = merged = 0
    for trial in range(320):
        init = [rng.standard_normal(size).astype(np.float32) for _ in range(nbuf)]
        keys = [plugin.tensor(a) for a in init]
        commands, spec = [], []
        for _ in range(int(rng.integers(2, 6))):
            kind = ["ADD", "MUL", "COPY"][int(rng.integers(0, 3))]
            ins = []
            for _side in range(2):
                k = int(rng.integers(0, nbuf))
                form = int(rng.integers(0, 4))
                if form <= 1:         # a window at a row offset
                    off = int(rng.integers(0, 4)) * width
                    ins.append((k, (rows, width), off, (width, 1)))
                elif form == 2:       # one row broadcast over the rows
                    off = int(rng.integers(0, rows)) * width
                    ins.append((k, (rows, width), off, (0, 1)))
                else:                 # one element broadcast everywhere
                    off = int(rng.integers(0, span))
                    ins.append((k, (rows, width), off, (0, 0)))
            ko = int(rng.integers(0, nbuf))
            oo = int(rng.integers(0, 4)) * width
            spec.append((kind, ins[0], ins[1], (ko, (rows, width), oo)))
            left = plugin.view(keys[ins[0][0]], ins[0][1], ins[0][2], list(ins[0][3]))
            right = plugin.view(keys[ins[1][0]], ins[1][1], ins[1][2], list(ins[1][3]))
            out = plugin.view(keys[ko], (rows, width), oo)
            if kind == "COPY":
                commands.append(("COPY", "copy", {"input": left, "output": out}))
            else:
                commands.append(binary(kind, left, right, out))
        status, _ = plugin.execute(commands)
        if status == m3.OK:
            expect = [a.copy() for a in init]
            _emulate(expect, spec)
            for k, e in zip(keys, expect):
                assert np.array_equal(bits(plugin.read(k)), bits(e)), (trial, spec)
            checked += 1
            merged += plugin.launches() < len(commands)
        else:
            # the reference rejects a command whose output overlaps its own
            # input in part; nothing may have been written
            for k, a in zip(keys, init):
                assert np.array_equal(bits(plugin.read(k)), bits(a))
        for k in keys:
            plugin.lib.m3_cuda_backend_free_storage(plugin.context, plugin.storages[k],
                                                    plugin.storages[k])
            del plugin.storages[k]
    assert checked >= 50 and merged >= 20, (checked, merged)


def _row_commands(plugin, kx, rows, width, kp, kv, ki, ks, order):
    x = plugin.view(kx, (rows, width))
    parts = {
        "SOFTMAX": ("SOFTMAX", "softmax", {"input": x, "output": plugin.view(kp, (rows, width))}),
        "TOP_K": ("TOP_K", "top_k", {"logits": x, "values": plugin.view(kv, (rows, 1)),
                                     "indices": plugin.view(ki, (rows, 1), dtype=plugin.m3.I32),
                                     "k": 1}),
        "ROW_SUM": ("ROW_SUM", "copy", {"input": x, "output": plugin.view(ks, (rows, 1))}),
    }
    return [parts[name] for name in order]


@pytest.mark.parametrize("rows,width", [(4096, 1024), (37, 300)])
def test_softmax_topk_rowsum_share_one_pass(m3, plugin, rows, width):
    """SOFTMAX, TOP_K and ROW_SUM of one input in one list: one NaN scan and
    one row pass, every output equal to running the commands one list each."""
    rng = np.random.default_rng(rows)
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
    kx = plugin.tensor(x)
    outs = [plugin.tensor(np.zeros(n, np.float32)) for n in (rows * width, rows, rows, rows)]
    order = ["SOFTMAX", "TOP_K", "ROW_SUM"]
    status, message = plugin.execute(_row_commands(plugin, kx, rows, width, *outs, order))
    assert status == m3.OK, message
    assert plugin.launches() == 2
    fused = [plugin.read(k) for k in outs]
    alone = [plugin.tensor(np.zeros(n, np.float32)) for n in (rows * width, rows, rows, rows)]
    for name in order:
        status, message = plugin.execute(_row_commands(plugin, kx, rows, width, *alone, [name]))
        assert status == m3.OK, message
    for got, k in zip(fused, alone):
        assert np.array_equal(bits(got), bits(plugin.read(k)))


def test_fused_rows_fail_atomically_and_in_command_order(m3, plugin):
    """A NaN in the input: SOFTMAX and TOP_K, merged, both stay untouched with
    the reference's message; a ROW_SUM listed before them is written first,
    as the reference's command-by-command order does."""
    rows, width = 64, 1024
    x = np.ones((rows, width), np.float32)
    x[40, 3] = np.nan
    kx = plugin.tensor(x)
    sentinel = np.float32(-7.0)
    outs = [plugin.tensor(np.full(n, sentinel, np.float32)) for n in (rows * width, rows, rows, rows)]
    status, message = plugin.execute(
        _row_commands(plugin, kx, rows, width, *outs, ["SOFTMAX", "TOP_K", "ROW_SUM"]))
    assert status == m3.OUT_OF_RANGE and message == "softmax input contains NaN"
    for k in outs:
        assert (plugin.read(k) == sentinel).all()
    status, message = plugin.execute(
        _row_commands(plugin, kx, rows, width, *outs, ["ROW_SUM", "TOP_K", "SOFTMAX"]))
    assert status == m3.OUT_OF_RANGE and message == "top-k logits contain NaN"
    sums = plugin.read(outs[3])
    assert sums[0] == np.float32(width) and np.isnan(sums[40])
    for k in outs[:3]:
        assert (plugin.read(k) == sentinel).all()


def _reference_outputs(m3, ref, build, inputs):
    """The reference's CPU provider on `build`'s graph."""
    g = m3.Graph(lib=ref)
    handles, outputs = build(g)
    s = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
    for name, vid in handles.items():
        s.write(vid, inputs[name])
    s.run()
    out = [s.read(v).copy() for v in outputs]
    s.close()
    return out


def test_vocoder_final_stage_in_command_order(m3, ref, plugin):
    """The vocoder's final stage in the reference's command order
    (src/m3_vocoder_decode.c:395-432): SNAKE1D into the activation buffer,
    CONV1D into the mono waveform, TANH in place on it.  No convolution runs
    on the GPU here, so the convolution is an opaque producer between two
    plug-in lists: computed on the host and written into the device storage,
    as the reference's m3_storage_write would.  The snake and the in-place
    tanh match the reference's CPU provider on the same inputs (the tanh on
    the same convolution output) within 2^-19, the bound of every
    transcendental here."""
    tol = 2.0 ** -19
    rng = np.random.default_rng(395)
    channels, length = 24, 3000
    hidden = (rng.standard_normal((2, channels, length)) * 0.5).astype(np.float32)
    alpha = rng.uniform(0.2, 2.0, (1, channels, 1)).astype(np.float32)
    weight = (rng.standard_normal((channels, 7)) * 0.2).astype(np.float64)
    kh, ka = plugin.tensor(hidden), plugin.tensor(alpha)
    kact = plugin.tensor(np.zeros_like(hidden))
    kmono = plugin.tensor(np.zeros((2, 1, length), np.float32))
    status, message = plugin.execute([("SNAKE1D", "snake1d", {
        "input": plugin.view(kh, hidden.shape), "alpha": plugin.view(ka, alpha.shape),
        "output": plugin.view(kact, hidden.shape)})])
    assert status == m3.OK, message
    activated = plugin.read(kact).reshape(hidden.shape)

    # the opaque producer: a 7-tap convolution, padding 3, to one channel
    padded = np.pad(activated.astype(np.float64), ((0, 0), (0, 0), (3, 3)))
    mono = np.zeros((2, 1, length))
    for c in range(channels):
        for k in range(7):
            mono[:, 0, :] += weight[c, k] * padded[:, c, k:k + length]
    mono = (mono * 0.25 + 0.01).astype(np.float32)
    plugin.write(kmono, mono)
    status, message = plugin.execute([("TANH", "tanh", {
        "input": plugin.view(kmono, mono.shape), "output": plugin.view(kmono, mono.shape)})])
    assert status == m3.OK, message
    waveform = plugin.read(kmono).reshape(mono.shape)

    def snake(g):
        vx = g.value(m3.INPUT, m3.F32, hidden.shape)
        va = g.value(m3.INPUT, m3.F32, alpha.shape)
        z = g.inferred("SNAKE1D", [vx, va], m3.OUTPUT, m3.F32)
        g.node("SNAKE1D", [vx, va], [z])
        return {"x": vx, "a": va}, [z]

    def tanh(g):
        vx = g.value(m3.INPUT, m3.F32, mono.shape)
        t = g.inferred("TANH", [vx], m3.OUTPUT, m3.F32)
        g.node("TANH", [vx], [t])
        return {"x": vx}, [t]

    (want_act,) = _reference_outputs(m3, ref, snake, {"x": hidden, "a": alpha})
    (want_wave,) = _reference_outputs(m3, ref, tanh, {"x": mono})
    for got, want in ((activated, want_act), (waveform, want_wave)):
        diff = np.abs(got.astype(np.float64) - want)
        assert ((diff <= tol) | (diff <= tol * np.abs(want))).all(), diff.max()
    assert np.abs(waveform).max() < 1.0 and np.abs(mono).max() > 0.5   # the tanh did work


def test_caller_stream_and_address_storages(m3, gpu):
    """A context on a caller's stream whose storage handles are device
    addresses (m3_cuda_backend_set_stream, m3_cuda_storage_is_address): the
    merged C1 chain computes the same bits as on the context's own stream,
    and the call has finished when it returns."""
    import torch

    lib = m3.load()
    err = m3.M3Error()
    accessor = ctypes.cast(lib.m3_cuda_storage_is_address, m3.STORAGE_DATA)
    context = ctypes.c_void_p()
    m3.check(lib.m3_cuda_backend_context_create(
        ctypes.byref(m3.BackendOptions(0, accessor, False)), ctypes.byref(context),
        ctypes.byref(err)), err)
    rows, width = 32, 256
    rng = np.random.default_rng(8)
    x = torch.from_numpy(rng.uniform(-1, 1, (rows, width)).astype(np.float32)).cuda()
    c = torch.from_numpy(rng.uniform(0.5, 2, width).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(width).astype(np.float32)).cuda()
    outs = {}
    stream = torch.cuda.Stream()
    try:
        for name, handle in (("caller", stream.cuda_stream), ("own", None)):
            m3.check(lib.m3_cuda_backend_set_stream(context, handle, ctypes.byref(err)), err)
            t, y = torch.zeros_like(x), torch.zeros_like(x)
            views = []

            def view(tensor, shape):
                v = m3.TensorView()
                v.metadata.dtype = m3.F32
                v.metadata.rank = len(shape)
                step = 4
                for axis in reversed(range(len(shape))):
                    v.metadata.shape[axis] = shape[axis]
                    v.byte_strides[axis] = step
                    step *= shape[axis]
                v.metadata.element_count = int(np.prod(shape))
                v.metadata.byte_count = v.metadata.element_count * 4
                v.storage = tensor.data_ptr()
                views.append(v)
                return ctypes.pointer(v)

            cmd = (m3.Command * 2)()
            cmd[0].kind, cmd[1].kind = m3.OPS["MUL"], m3.OPS["ADD"]
            cmd[0].descriptor.mul.left = view(x, (rows, width))
            cmd[0].descriptor.mul.right = view(c, (width,))
            cmd[0].descriptor.mul.output = view(t, (rows, width))
            cmd[1].descriptor.add.left = view(t, (rows, width))
            cmd[1].descriptor.add.right = view(b, (1, width))
            cmd[1].descriptor.add.output = view(y, (rows, width))
            torch.cuda.synchronize()
            m3.check(lib.m3_cuda_backend_execute(context, cmd, 2, None, ctypes.byref(err)), err)
            assert lib.m3_cuda_backend_launch_count(context) == 1
            outs[name] = y.cpu().numpy()    # no wait needed: execute has returned
    finally:
        lib.m3_cuda_backend_destroy_context(context)
    want = x.cpu().numpy() * c.cpu().numpy() + b.cpu().numpy()
    for got in outs.values():
        assert np.array_equal(bits(got), bits(want))
