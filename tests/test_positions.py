"""The ring's host-side ordering board (`ce_transport._Positions`) on two CPU
ranks over gloo: a rank sees what its peer published, a wait for a position
nobody publishes raises within FPEMU_HOST_WAIT_S instead of hanging, and the
shared-memory blocks are cleaned up by their owners only -- no process's
resource tracker reports a leaked or missing block at exit.  The ranks run in a
child interpreter so that its whole stderr, resource trackers included, can be
inspected."""
from __future__ import annotations

import socket
import subprocess
import sys
import textwrap

from conftest import REPO

_SCRIPT = textwrap.dedent(
    """
    import os, sys
    from datetime import timedelta
    import torch.multiprocessing as mp

    def worker(rank, port, q):
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), FPEMU_HOST_WAIT_S="0.3")
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=30))
        from fp_emulation.ce_transport import _Positions
        board = _Positions(dist.group.WORLD, rank, 2, "test")
        out = []
        if rank == 0:
            board.publish(5)
        dist.barrier()
        if rank == 1:
            board.wait(0, 5, "published item")
            out.append("saw 5")
            try:
                board.wait(0, 6, "unpublished item")
                out.append("no timeout")
            except RuntimeError as exc:
                out.append("timeout" if "did not enqueue unpublished item" in str(exc) else repr(exc))
        dist.barrier()
        board.close()
        dist.destroy_process_group()
        q.put((rank, out))

    if __name__ == "__main__":
        sys.path[:0] = [{pkg!r}, {repo!r}]
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        port = int(sys.argv[1])
        ps = [ctx.Process(target=worker, args=(r, port, q)) for r in range(2)]
        for p in ps:
            p.start()
        res = dict(q.get(timeout=120) for _ in ps)
        for p in ps:
            p.join(timeout=60)
        print(res[1])
        sys.exit(0 if all(p.exitcode == 0 for p in ps) else 1)
    """
)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_positions_board_orders_times_out_and_cleans_up(tmp_path):
    script = tmp_path / "board.py"
    script.write_text(_SCRIPT.format(pkg=str(REPO / "fp-emulation_b200"), repo=str(REPO)))
    out = subprocess.run([sys.executable, str(script), str(_free_port())], capture_output=True, text=True,
                         timeout=300, env={"PYTHONPATH": str(REPO / "fp-emulation_b200"), "PATH": "/usr/bin:/bin"})
    assert out.returncode == 0, out.stderr[-3000:]
    assert out.stdout.strip().splitlines()[-1] == "['saw 5', 'timeout']"
    assert "resource_tracker" not in out.stderr, out.stderr[-3000:]


def test_board_block_replaces_a_stale_file(tmp_path):
    """A block left by a dead process with the same pid is replaced, not an error."""
    import numpy as np

    from fp_emulation.ce_transport import _Positions

    path = tmp_path / "fpemu_pos_stale"
    path.write_bytes(b"\xff" * 8)
    m = _Positions._map(str(path), create=True)
    np.ndarray((1,), dtype=np.int64, buffer=m)[0] = 7
    peer = _Positions._map(str(path))
    assert int(np.ndarray((1,), dtype=np.int64, buffer=peer)[0]) == 7
    peer.close()
    m.close()
