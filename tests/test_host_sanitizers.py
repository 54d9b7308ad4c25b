"""The native host runtime (paged-KV bookkeeping, VRAM arena, RAM pool) built with AddressSanitizer and
UndefinedBehaviorSanitizer, driven through random operation sequences in a child process:
a heap error or undefined behaviour aborts the child, and every sequence must return all of
its blocks to the pool when freed."""
import os
import shutil
import subprocess
import sys
import sysconfig

import pytest

ROOT = os.path.join(os.path.dirname(__file__), "..")

DRIVER = r"""
import random, sys
sys.path.insert(0, sys.argv[1])
import _host
for seed in range(4):
    random.seed(seed)
    m = _host.SequenceManager(24, 4)
    live = []
    for i in range(5000):
        op = random.choice("cafts ix")
        try:
            if op == "c":
                live.append(m.create_sequence())
            elif live:
                s = random.choice(live)
                if op == "a": m.append(s, random.randint(1, 9))
                elif op == "f": live.append(m.fork_sequence(s))
                elif op == "t": m.truncate(s, random.randint(0, m.num_tokens(s)))
                elif op == "s": m.swap_out(s)
                elif op == "i": m.swap_in(s)
                elif op == "x": live.remove(s); m.free_sequence(s)
                elif op == " ": m.cow_last_block(s)
        except (RuntimeError, ValueError, IndexError):
            pass
    for s in live:
        m.free_sequence(s)
    assert m.allocator.num_free_blocks() == 24, m.allocator.num_free_blocks()
for seed in range(4):
    random.seed(seed)
    a = _host.VramArena(1 << 20, 4096)
    held = []
    for i in range(3000):
        if held and random.random() < 0.45:
            a.free(held.pop(random.randrange(len(held))))
        else:
            x = a.allocate(random.randint(1, 50000), random.choice([1, 256, 4096]))
            if x is not None:
                held.append(x)
    for x in held:
        a.free(x)
    assert a.used == 0 and a.fragment_count() == 1 and a.largest_free() == a.usable
    pool = _host.RamPool(1 << 18)
    bufs = [pool.acquire(random.randint(1, 70000)) for _ in range(64)]
    for b in bufs:
        memoryview(b)[:len(b)] = b"x" * len(b)
        pool.release(b)
print("clean")
"""


def _lib(name):
    p = subprocess.run(["g++", f"-print-file-name={name}"], capture_output=True, text=True).stdout.strip()
    return p if os.path.isabs(p) and os.path.exists(p) else None


@pytest.mark.skipif(shutil.which("g++") is None or _lib("libasan.so") is None, reason="needs g++ with ASan")
def test_host_runtime_under_asan_ubsan(tmp_path):
    import pybind11
    out = tmp_path / ("_host" + sysconfig.get_config_var("EXT_SUFFIX"))
    src = [os.path.join(ROOT, "csrc", "host", f) for f in ("host_kv.cpp", "arena.cpp", "module.cpp")]
    cmd = ["g++", "-shared", "-fPIC", "-O1", "-g", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
           "-std=c++17", "-DAIR_HOST_NO_TORCH", "-I" + pybind11.get_include(),
           "-I" + sysconfig.get_paths()["include"], *src, "-o", str(out)]
    subprocess.run(cmd, check=True, capture_output=True, timeout=600)
    env = dict(os.environ, LD_PRELOAD=":".join(x for x in (_lib("libasan.so"), _lib("libubsan.so")) if x),
               ASAN_OPTIONS="detect_leaks=0:abort_on_error=1", UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([sys.executable, "-c", DRIVER, str(tmp_path)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "clean" in r.stdout, r.stderr[-3000:]
