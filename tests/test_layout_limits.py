"""The shared-memory layout of the tensor-memory multi-query kernel against the limit the
header promises (no GPU: the layout function is host code, compiled here with nvcc).

gollek_paged_attention_v2 serves 32 and 64 q heads per kv head on prefill_tc_kernel, whose
per-CTA shared memory grows with the number of sequences in the call (their prefix sums
and lengths).  The host tries, in order, the two-warp form and then the one-warp form,
each with K/V rings {2,3}, {2,2}, {1,2}, within 227 KB.  The header states the largest
sequence count that fits; this test recomputes it for a 148-SM B200, and checks that the
benchmarked case (64 sequences) gets the two-warp form with the deepest rings.
"""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROG = r"""
#include <cstdio>
#include <cudaTypedefs.h>
#include "prefill_tc.cuh"
int main() {
    const int rings[3][2] = {{2, 3}, {2, 2}, {1, 2}};
    for (int nq : {32, 64})
        for (int h = 0; h < 2; ++h) {
            int best = 0;
            for (int S = 1; S < 20000; ++S)
                for (const auto &r : rings)
                    if (gk::pt_smem_layout(nq, r[0], r[1], S, 148, h).total <= 227 * 1024) {
                        best = S;
                        break;
                    }
            printf("max %d %d %d\n", nq, h, best);
        }
    for (int nq : {32, 64})
        printf("bench %d %u\n", nq, gk::pt_smem_layout(nq, 2, 3, 64, 148, true).total);
    return 0;
}
"""


@pytest.fixture(scope="module")
def limits(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    d = tmp_path_factory.mktemp("layout")
    (d / "t.cu").write_text(PROG)
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
                    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "gollek_b200", "csrc"),
                    "-I", os.path.join(ROOT, "include"), "-o", str(d / "t"), str(d / "t.cu")],
                   check=True, capture_output=True, timeout=300)
    out = subprocess.run([str(d / "t")], check=True, capture_output=True, text=True).stdout
    mx = {(int(a), int(b)): int(c) for a, b, c in re.findall(r"max (\d+) (\d+) (\d+)", out)}
    bench = {int(a): int(b) for a, b in re.findall(r"bench (\d+) (\d+)", out)}
    return mx, bench


def test_header_sequence_limit(limits):
    mx, _ = limits
    text = open(os.path.join(ROOT, "include", "gollek_kernels.h")).read()
    m = re.search(r"up to ([\d,]+) sequences per call", text)
    assert m, "the header states the sequence limit of 32- and 64-head groups"
    promised = int(m.group(1).replace(",", ""))
    # a call runs whichever form fits; the binding group size is the larger one
    assert min(max(mx[(nq, 0)], mx[(nq, 1)]) for nq in (32, 64)) == promised
    # the two-warp form's hand-over area costs a few sequences: the fallback keeps them
    assert mx[(64, 1)] < mx[(64, 0)] and mx[(32, 1)] < mx[(32, 0)]


def test_benchmarked_case_gets_two_warps_and_deep_rings(limits):
    _, bench = limits
    for nq in (32, 64):
        assert bench[nq] <= 227 * 1024
