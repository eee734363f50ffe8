"""The expert server's stdin/stdout protocol (npu-kernels/npu_kernels/rngd/template/src/bin/server.rs.tpl:1-8,
63-97): LOAD / RUN / UPDATE / RUN_WSUM / EXIT framing on the CPU with a backend computing rows with the
oracle, and the real server process on a GPU, driven through a pipe, against the oracle."""
import io
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from npu_offload_b200 import expert_server as xs
from npu_offload_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _experts(seed, E, H, F):
    return [synth.expert_weights(seed, 0, e, H, F) for e in range(E)]


def _write_tables(base, experts):
    """<base>.g / .u / .d: the slots back to back, row-major bf16."""
    np.concatenate([g.ravel() for g, _, _ in experts]).astype("<u2").tofile(base + ".g")
    np.concatenate([u.ravel() for _, u, _ in experts]).astype("<u2").tofile(base + ".u")
    np.concatenate([d.ravel() for _, _, d in experts]).astype("<u2").tofile(base + ".d")


def _oracle_rows(experts, slots, x):
    from oracle.oracle import Port
    rows = []
    for s in slots:
        g, u, d = experts[s]
        rows.append(Port.cpu_moe(x[None], [("bf16", np.concatenate([g, u], 0), d)], [[0]], [[1.0]])[0])
    return np.stack(rows)


class OracleBackend:
    """Rows from the C restatement (CPU): exercises the protocol without a GPU."""

    def __init__(self, H, F, E, K, L):
        self.H, self.F, self.E, self.K, self.L = H, F, E, K, L
        self.tables = {}

    def loaded(self, layer):
        return layer in self.tables

    def load(self, layer, g, u, d):
        self.tables[layer] = [(g[e].copy(), u[e].copy(), d[e].copy()) for e in range(self.E)]

    def update(self, layer, slot, g, u, d):
        self.tables[layer][slot] = (g.copy(), u.copy(), d.copy())

    def rows(self, layer, slots, x):
        return _oracle_rows(self.tables[layer], slots, x)


def _req(*fields):
    return b"".join(f if isinstance(f, bytes) else struct.pack("<I", f) for f in fields)


def _path_field(p):
    b = p.encode()
    return _req(len(b), b)


def test_protocol_round_trip_on_cpu(tmp_path):
    H, F, E, K, L = 128, 64, 6, 4, 2
    ex = _experts(3, E, H, F)
    _write_tables(str(tmp_path / "l0"), ex)
    new = _experts(9, 1, H, F)
    _write_tables(str(tmp_path / "s2"), new)
    x = synth.hidden(4, 1, H)[0]
    w = np.array([0.5, 0.25, 0.125], np.float32)
    inp = io.BytesIO(b"".join([
        _req(xs.OP_LOAD, 0), _path_field(str(tmp_path / "l0")),
        _req(xs.OP_RUN, 0, 3, 1, 4, 2), x.astype("<u2").tobytes(),
        _req(xs.OP_RUN_WSUM, 0, 3, 1, 4, 2), w.astype("<f4").tobytes(), x.astype("<u2").tobytes(),
        _req(xs.OP_UPDATE, 0, 2), _path_field(str(tmp_path / "s2")),
        _req(xs.OP_RUN, 0, 1, 2), x.astype("<u2").tobytes(),
        _req(xs.OP_LOAD, 5), _path_field(str(tmp_path / "l0")),          # layer out of range
        _req(xs.OP_LOAD, 1), _path_field(str(tmp_path / "missing")),     # no such file
        _req(xs.OP_UPDATE, 0, 9), _path_field(str(tmp_path / "s2")),     # slot out of range
        _req(77),                                                         # unknown op
        _req(xs.OP_EXIT),
    ]))
    out = io.BytesIO()
    assert xs.serve_stream(inp, out, OracleBackend(H, F, E, K, L)) == 0
    r = io.BytesIO(out.getvalue())
    assert r.read(4) == b"RDY1"
    assert struct.unpack("<I", r.read(4))[0] == xs.ST_OK
    rows = np.frombuffer(r.read(3 * H * 2), "<u2").reshape(3, H)
    ref = _oracle_rows(ex, [1, 4, 2], x)
    np.testing.assert_array_equal(rows, xs.f2bf(ref))
    wsum = np.frombuffer(r.read(H * 4), "<f4")
    acc = np.zeros(H, np.float32)
    for k in range(3):
        acc += w[k] * ref[k]
    np.testing.assert_array_equal(wsum, acc)
    assert struct.unpack("<I", r.read(4))[0] == xs.ST_OK
    row2 = np.frombuffer(r.read(H * 2), "<u2")
    np.testing.assert_array_equal(row2, xs.f2bf(_oracle_rows(new, [0], x))[0])
    assert struct.unpack("<4I", r.read(16)) == (xs.ST_BAD_INDEX, xs.ST_BAD_FILE, xs.ST_BAD_INDEX, xs.ST_UNKNOWN)
    assert r.read() == b""


def test_run_on_an_unloaded_layer_is_a_protocol_error():
    H, F, E, K, L = 64, 64, 2, 2, 1
    inp = io.BytesIO(_req(xs.OP_RUN, 0, 1, 0) + np.zeros(H, "<u2").tobytes())
    with pytest.raises(xs.ProtocolError):
        xs.serve_stream(inp, io.BytesIO(), OracleBackend(H, F, E, K, L))
    inp = io.BytesIO(_req(xs.OP_RUN, 0, K + 1))
    with pytest.raises(xs.ProtocolError):
        xs.serve_stream(inp, io.BytesIO(), OracleBackend(H, F, E, K, L))


def test_end_of_input_ends_the_server():
    out = io.BytesIO()
    assert xs.serve_stream(io.BytesIO(b""), out, OracleBackend(64, 64, 2, 2, 1)) == 0
    assert out.getvalue() == b"RDY1"


@pytest.mark.gpu
def test_server_process_through_a_pipe_matches_oracle(tmp_path):
    """The server as a process (python -m npu_offload_b200.expert_server), Solar-shaped H and F with
    E = 8 slots: LOAD, RUN of 8 slots, RUN_WSUM, UPDATE of one slot, RUN again, EXIT."""
    from tests.parity import assert_close
    H, F, E, K = 4096, 1280, 8, 8
    ex = _experts(11, E, H, F)
    _write_tables(str(tmp_path / "layer0"), ex)
    new = _experts(12, 1, H, F)
    _write_tables(str(tmp_path / "slot5"), new)
    x = synth.hidden(13, 1, H)[0]
    slots = [7, 0, 5, 3, 1, 6, 2, 4]
    w = np.linspace(0.05, 0.3, 8).astype(np.float32)
    p = subprocess.Popen([sys.executable, "-m", "npu_offload_b200.expert_server", "--hidden", str(H), "--inter",
                          str(F), "--experts", str(E), "--top-k", str(K), "--layers", "2"],
                         stdin=subprocess.PIPE, stdout=subprocess.PIPE, cwd=ROOT)
    try:
        assert p.stdout.read(4) == b"RDY1"

        def call(data, nbytes):
            p.stdin.write(data)
            p.stdin.flush()
            return p.stdout.read(nbytes)

        assert struct.unpack("<I", call(_req(xs.OP_LOAD, 1) + _path_field(str(tmp_path / "layer0")), 4))[0] == 0
        rows = np.frombuffer(call(_req(xs.OP_RUN, 1, 8, *slots) + x.astype("<u2").tobytes(), 8 * H * 2), "<u2")
        ref = _oracle_rows(ex, slots, x)
        from oracle.oracle import bf2f
        assert_close(bf2f(rows.reshape(8, H)), ref, what="RUN rows vs oracle")
        wsum = np.frombuffer(call(_req(xs.OP_RUN_WSUM, 1, 8, *slots) + w.astype("<f4").tobytes()
                                  + x.astype("<u2").tobytes(), H * 4), "<f4")
        assert_close(wsum, (w[:, None] * ref).sum(0), what="RUN_WSUM vs oracle")
        assert struct.unpack("<I", call(_req(xs.OP_UPDATE, 1, 5) + _path_field(str(tmp_path / "slot5")), 4))[0] == 0
        row5 = np.frombuffer(call(_req(xs.OP_RUN, 1, 1, 5) + x.astype("<u2").tobytes(), H * 2), "<u2")
        assert_close(bf2f(row5)[None], _oracle_rows(new, [0], x), what="RUN after UPDATE vs oracle")
        p.stdin.write(_req(xs.OP_EXIT))
        p.stdin.flush()
        assert p.wait(timeout=60) == 0
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()
