"""The hot-expert server's mailbox protocol (track2_opt/expert_srv/src/main.rs:1-20, client
solar_hybrid/opt_client.py): host logic on the CPU, and the served rows on a GPU against the oracle."""
import os
import struct
import subprocess
import sys
import time

import numpy as np
import pytest

from npu_offload_b200 import expert_srv as es
from npu_offload_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _pack(slots):
    """The client's id word (opt_client.OptExpertServer.ffn)."""
    p = len(slots) << 56
    for k, e in enumerate(slots):
        p += e << (6 * k)
    return p


def test_packed_ids_round_trip():
    for slots in ([0], [31, 0, 5], list(range(24, 32))):
        assert es.unpack_ids(_pack(slots)) == (len(slots), slots)


def test_layer_file_layout(tmp_path):
    H, F = 64, 32
    rng = np.random.default_rng(0)
    parts, ref = [], []
    for e in range(es.E_SRV):
        g, u, d = (rng.integers(0, 65535, size=s, dtype=np.uint16) for s in ((F, H), (F, H), (H, F)))
        parts += [g.ravel(), u.ravel(), d.ravel()]  # [Wg][Wu][Wd] per slot (opt_client.export_tables)
        ref.append((g, u, d))
    p = tmp_path / "layer_0.bin"
    np.concatenate(parts).tofile(p)
    got = es.load_layer_file(str(p), H, F)
    for (a, b, c), (x, y, z) in zip(got, ref):
        np.testing.assert_array_equal(a, x)
        np.testing.assert_array_equal(b, y)
        np.testing.assert_array_equal(c, z)
    with pytest.raises(ValueError):
        es.load_layer_file(str(p), H, F + 32)


def _request(mm, seq, op, layer, packed, timeout=60.0):
    struct.pack_into("<IIQ", mm, 16, op, layer, packed)
    struct.pack_into("<Q", mm, 0, seq)
    t0 = time.time()
    while struct.unpack_from("<Q", mm, 8)[0] != seq:
        if time.time() - t0 > timeout:
            raise TimeoutError("server did not answer")
        time.sleep(0)
    return struct.unpack_from("<I", mm, 32)[0]


@pytest.mark.gpu
def test_server_rows_match_oracle(tmp_path):
    import mmap
    from oracle.oracle import Port, bf2f
    from tests.parity import assert_close
    H, F, L = 1024, 256, 2
    W = [[synth.expert_weights(8, l, e, H, F) for e in range(es.E_SRV)] for l in range(L)]
    for l in range(L):
        np.concatenate([a.ravel() for e in W[l] for a in e]).tofile(tmp_path / f"layer_{l}.bin")
    shm = tmp_path / "mailbox"
    with open(shm, "wb") as f:
        f.write(b"\0" * es.shm_bytes(H))
    proc = subprocess.Popen([sys.executable, "-m", "npu_offload_b200.expert_srv", str(shm), str(tmp_path), str(L),
                             "--hidden", str(H), "--inter", str(F)], cwd=ROOT)
    f = open(shm, "r+b")
    mm = mmap.mmap(f.fileno(), es.shm_bytes(H))
    x_view = out_view = None
    try:
        t0 = time.time()
        while struct.unpack_from("<I", mm, 36)[0] != 1:
            assert proc.poll() is None, "server exited"
            assert time.time() - t0 < 300, "server not ready"
            time.sleep(0.2)
        x_view = np.frombuffer(mm, dtype=np.uint16, count=H, offset=es.OFF_X)
        out_view = np.frombuffer(mm, dtype=np.uint16, count=es.K_MAX * H, offset=es.OFF_OUT)
        seq = 0
        for layer, slots in ((1, [3, 31, 0, 7, 12, 5, 20, 9]), (0, [17]), (0, [2, 2, 30])):
            x = synth.hidden(100 + layer + len(slots), 1, H)[0]
            x_view[:] = x
            seq += 1
            assert _request(mm, seq, 1, layer, _pack(slots)) == 0
            rows = out_view[:len(slots) * H].reshape(len(slots), H).copy()
            for k, s in enumerate(slots):
                g, u, d = W[layer][s]
                ref = Port.cpu_moe(x[None], [("bf16", np.concatenate([g, u], 0), d)], [[0]], [[1.0]])[0]
                assert_close(bf2f(rows[k]), ref, what=f"layer {layer} slot {s}")
        assert struct.unpack_from("<d", mm, 40)[0] > 0  # last_us
        seq += 1
        assert _request(mm, seq, 1, L, _pack([0])) == 2  # bad layer
        seq += 1
        assert _request(mm, seq, 1, 0, _pack([40])) == 3  # bad slot
        seq += 1
        assert _request(mm, seq, 7, 0, 0) == 1  # unknown op
        seq += 1
        _request(mm, seq, 3, 0, 0)  # quit
        assert proc.wait(timeout=60) == 0
    finally:
        if proc.poll() is None:
            proc.kill()
        del x_view, out_view  # release the buffer exports before unmapping
        mm.close()
        f.close()
