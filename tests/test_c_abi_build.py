"""The C ABI as a C or C++ host sees it: a program that includes include/hmb.h, compiled as C99 and as
C++17 and linked against heteromega_b200/libhmb.so, runs the host-side entry points (no GPU needed):
packing a matrix, the tile index, the slice tile counts, the status strings. The packed bytes must
equal the Python packer's, which the golden tests pin to the reference's packers."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

import heteromega_b200 as H

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(REPO, "heteromega_b200")

PROGRAM = r"""
#include <stdio.h>
#include <stdlib.h>
#include "hmb.h"

int main(void) {
    const int64_t k = 256, n = 192;
    uint8_t *q = (uint8_t *)malloc(k * n), *z = (uint8_t *)malloc((k / 128) * n);
    uint16_t *s = (uint16_t *)malloc((k / 128) * n * 2);
    for (int64_t i = 0; i < k * n; ++i) q[i] = (uint8_t)((i * 7 + 3) % 16);
    for (int64_t i = 0; i < (k / 128) * n; ++i) { z[i] = (uint8_t)(i % 16); s[i] = (uint16_t)(0x3C00 + i % 97); }
    const int64_t bytes = hmb_packed_bytes(k, n);
    uint8_t *out = (uint8_t *)malloc(bytes);
    if (hmb_version() <= 0 || bytes != 2 * 3 * HMB_TILE_BYTES) return 2;
    if (hmb_pack_w4a16(q, s, z, k, n, out) != HMB_OK) return 3;
    q[5] = 16;
    if (hmb_pack_w4a16(q, s, z, k, n, out + 0) != HMB_ERR_VALUE) return 4;
    int64_t gu = 0, dn = 0;
    if (hmb_slice_tile_counts(1024, 4096, 128, 640, &gu, &dn) != HMB_OK) return 5;
    printf("%lld %lld %lld %s\n", (long long)hmb_packed_tile_index(2, 1, 2, 3), (long long)gu, (long long)dn,
           hmb_status_string(HMB_ERR_TIMEOUT));
    q[5] = (uint8_t)((5 * 7 + 3) % 16);
    hmb_pack_w4a16(q, s, z, k, n, out);
    FILE *f = fopen(getenv("HMB_OUT"), "wb");
    fwrite(out, 1, (size_t)bytes, f);
    fclose(f);
    return 0;
}
"""


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_header_compiles_links_and_runs(tmp_path, lang):
    lib = os.path.join(LIBDIR, "libhmb.so")
    if not os.path.exists(lib):
        pytest.skip("libhmb.so is not built")
    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip(f"no {lang} compiler")
    src = tmp_path / ("prog.c" if lang == "c" else "prog.cpp")
    src.write_text(PROGRAM)
    exe = tmp_path / "prog"
    std = "-std=c99" if lang == "c" else "-std=c++17"
    subprocess.run([cc, std, "-Wall", "-Werror", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe), "-L", LIBDIR,
                    "-lhmb", f"-Wl,-rpath,{LIBDIR}"], check=True, capture_output=True)
    out_file = tmp_path / "packed.bin"
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=dict(os.environ, HMB_OUT=str(out_file)))
    assert r.returncode == 0, (r.returncode, r.stderr)
    tile_index, gu, dn, status = r.stdout.split(maxsplit=3)
    assert int(tile_index) == H.packed_tile_index(2, 1, 2, 3)
    assert (int(gu), int(dn)) == (8 * 16, 4 * 16)  # 512 channels: gate_up [1024, 1024], down [512, 1024]
    assert "wait" in status.lower() or "time" in status.lower()

    k, n = 256, 192
    i = np.arange(k * n)
    q = ((i * 7 + 3) % 16).astype(np.uint8).reshape(k, n)
    j = np.arange((k // 128) * n)
    z = (j % 16).astype(np.uint8).reshape(k // 128, n)
    s = (0x3C00 + j % 97).astype(np.int16).reshape(k // 128, n)
    ref = H.pack_w4a16(torch.from_numpy(q), torch.from_numpy(s).view(torch.bfloat16), torch.from_numpy(z))
    assert np.array_equal(np.fromfile(out_file, np.uint8), ref.numpy())
