"""Failure handling of the calibration exchange on the host, without a GPU: the library's NCCL
entry points are pointed (XSAKE_NCCL_LIBRARY) at a fake NCCL built here with gcc, whose
communicator never finishes initialising when more than one rank is asked for (a rank that
never joins).  xsake_comm_init_ex must return XSAKE_ETIMEOUT within its deadline and abort the
communicator; a one-rank communicator initialises, all-reduces and is destroyed.  Each case runs
in a child process (the NCCL library is chosen once per process)."""

import os
import shutil
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = r"""
#include <string.h>
typedef struct { char internal[128]; } ncclUniqueId;
typedef int ncclResult_t;
static int g_abort = 0, g_destroy = 0, g_nranks = 0;
static char g_comm;
int fake_aborts(void) { return g_abort; }
int fake_destroys(void) { return g_destroy; }
ncclResult_t ncclGetUniqueId(ncclUniqueId* id) { memset(id, 7, sizeof(*id)); return 0; }
ncclResult_t ncclCommInitRankConfig(void** c, int n, ncclUniqueId id, int r, void* cfg) {
  (void)id; (void)r; (void)cfg; g_nranks = n; *c = &g_comm; return 7;   /* ncclInProgress */
}
ncclResult_t ncclCommGetAsyncError(void* c, ncclResult_t* st) { (void)c; *st = g_nranks == 1 ? 0 : 7; return 0; }
ncclResult_t ncclAllReduce(const void* s, void* r, unsigned long n, int t, int op, void* c, void* st) {
  (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st; return 0;
}
ncclResult_t ncclCommAbort(void* c) { (void)c; ++g_abort; return 0; }
ncclResult_t ncclCommDestroy(void* c) { (void)c; ++g_destroy; return 0; }
const char* ncclGetErrorString(ncclResult_t r) { (void)r; return "fake nccl"; }
"""

CHILD = textwrap.dedent("""
    import ctypes as C, sys, time
    sys.path.insert(0, {root!r})
    from xsake_b200 import _lib, comm
    fake = C.CDLL({fake!r})
    lib = _lib.load()
    uid = comm.unique_id()
    t0 = time.monotonic()
    try:
        comm.Comm(uid, 2, 0, timeout_s=0.3)
        print("NO-TIMEOUT")
    except _lib.XsakeError as e:
        print("code", e.code, "elapsed", round(time.monotonic() - t0, 3), "aborts", fake.fake_aborts())
    c = comm.Comm(uid, 1, 0, timeout_s=0.3)
    assert lib.xsake_comm_allreduce_sum_f64(c._comm, None, 0, None) == 0
    c.destroy()
    print("single ok destroys", fake.fake_destroys(), "aborts", fake.fake_aborts())
""")


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("fake_nccl")
    src, so = d / "fake_nccl.c", d / "libfake_nccl.so"
    src.write_text(FAKE)
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so), str(src)], check=True)
    return str(so)


def test_rank_that_never_joins_times_out_and_aborts(fake_nccl):
    lib = os.path.join(ROOT, "xsake_b200", "lib", "libxsake_hads.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    env = dict(os.environ, XSAKE_NCCL_LIBRARY=fake_nccl)
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT, fake=fake_nccl)], env=env,
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    first, second = r.stdout.strip().splitlines()[-2:]
    words = first.split()
    assert words[0] == "code" and int(words[1]) == 4          # XSAKE_ETIMEOUT
    assert 0.3 <= float(words[3]) < 5.0                       # bounded by the deadline
    assert int(words[5]) == 1                                 # the communicator was aborted
    assert second.startswith("single ok destroys 1")
