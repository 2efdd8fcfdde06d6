"""The device's exp (vq3r_common.cuh expf_cr), used by the VQ4P expert loop
and by KDA, compiled for the host by nvcc and checked on the CPU: equal to
exp computed in double and rounded once (the correctly rounded result) on
a sample of floats across the whole range, and to glibc's expf — which the
reference's silu calls (src/model.c:501) — on all but a small fraction of
it (glibc's expf is within 0.502 ulp, so it differs only next to rounding
midpoints)."""
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "warp_b200", "csrc")

PROG = r"""
#include "vq3r_common.cuh"
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
int main() {
    unsigned long long n = 0, vs_cr = 0, vs_glibc = 0;
    for (uint32_t u = 0; u < 0xFFFFFFF0u; u += 613) {
        float x;
        memcpy(&x, &u, 4);
        if (!(x >= -110.0f && x <= 95.0f)) continue;
        const float a = wc::expf_cr(x), b = expf(x), c = (float)exp((double)x);
        n++;
        vs_cr += memcmp(&a, &c, 4) != 0;
        vs_glibc += memcmp(&a, &b, 4) != 0;
    }
    const float sp[] = {0.0f, -0.0f, -103.9f, -104.5f, 88.7f, 88.8f, 89.5f};
    for (float x : sp) {
        const float a = wc::expf_cr(x), c = (float)exp((double)x);
        n++;
        vs_cr += memcmp(&a, &c, 4) != 0;
    }
    printf("%llu %llu %llu\n", n, vs_cr, vs_glibc);
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not on PATH")
def test_expf_cr_is_correctly_rounded():
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "t.cu"), os.path.join(d, "t")
        with open(src, "w") as f:
            f.write(PROG)
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-I", CSRC, src, "-o", exe], check=True,
                       capture_output=True)
        n, vs_cr, vs_glibc = map(int, subprocess.run([exe], check=True, capture_output=True,
                                                     text=True).stdout.split())
    assert n > 5_000_000
    assert vs_cr == 0
    assert vs_glibc / n < 2e-4
