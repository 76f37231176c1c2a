"""gollek_b200.build under concurrent callers (the ranks of one job finding stale sources).

Each of four processes calls build() against a library path in a temporary directory whose
compile step is replaced by a slow stand-in that counts its runs: exactly one compile may
run, and every caller must return a complete file.
"""
import multiprocessing as mp
import os
import time


def _worker(libdir, barrier, q):
    from gollek_b200 import build as B
    B.LIB_DIR = libdir
    B.LIB_PATH = os.path.join(libdir, "libgollek_kernels.so")
    B.stale = lambda: not os.path.exists(B.LIB_PATH)

    def fake_compile(verbose):
        with open(os.path.join(libdir, "compiles"), "a") as f:
            f.write("x")
        tmp = f"{B.LIB_PATH}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            for _ in range(8):
                f.write(b"\0" * 4096)
                f.flush()
                time.sleep(0.05)
        os.replace(tmp, B.LIB_PATH)
        return B.LIB_PATH

    B._build_locked = fake_compile
    barrier.wait()
    path = B.build()
    q.put(os.path.getsize(path))


def test_one_compile_for_concurrent_callers(tmp_path):
    ctx = mp.get_context("spawn")
    barrier = ctx.Barrier(4)
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(str(tmp_path), barrier, q)) for _ in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    sizes = [q.get(timeout=10) for _ in procs]
    assert sizes == [8 * 4096] * 4
    assert open(tmp_path / "compiles").read() == "x"


def test_source_edited_during_a_build_reads_stale(tmp_path, monkeypatch):
    """A library whose build started before a source edit is stale, even though the edit
    happened before the build finished."""
    from gollek_b200 import build as B
    src = tmp_path / "k.cu"
    src.write_text("a")
    lib = tmp_path / "lib.so"
    monkeypatch.setattr(B, "LIB_PATH", str(lib))
    monkeypatch.setattr(B, "sources", lambda: [str(src)])
    real_run = B.subprocess.run

    def fake_run(cmd, **kw):
        out = cmd[cmd.index("-o") + 1]
        time.sleep(0.05)
        now = time.time()
        os.utime(src, (now, now))  # edited mid-build ...
        time.sleep(0.05)
        open(out, "wb").write(b"\0")  # ... before the output is written
        return real_run(["true"], **kw)

    monkeypatch.setattr(B.subprocess, "run", fake_run)
    B._build_locked(False)
    assert B.stale()
