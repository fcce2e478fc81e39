"""Host check of the K/V pool addressing shared by the kernels (tinyinfer_b200/csrc/kernels.h).

The forward context stores its pools layer-major while its API (COW regions,
mp_kv_read / mp_kv_write) speaks reference-layout offsets
([block][layer][slot][kv_width], miniprefix/include/miniprefix/paged_kv.h:25-27).
The COW kernel translates offsets with layer_major_offset(); the attention, append
and prefill kernels address pages with pool_page(). This compiles both helpers as
host code and checks, element by element on a small pool, that the translation is
a bijection, that it lands where pool_page() puts the same (block, layer, slot,
column), that a piece cut at reference page boundaries stays contiguous, and that
pool_page() with the reference strides reproduces the reference offsets.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INCLUDE = "/usr/local/cuda/include"

CHECKER = r"""
#include "kernels.h"
#include <cstdio>
#include <vector>

int main() {
    const int bt = 4, layers = 3, blocks = 5;
    const uint64_t page = uint64_t(bt) * mpb::kKvWidth, pool = page * layers * blocks;
    const mpb::PoolGeometry g{page, uint64_t(layers), uint64_t(blocks)};
    std::vector<char> hit(pool, 0);
    for (uint64_t e = 0; e < pool; ++e) {
        const uint64_t lm = mpb::layer_major_offset(g, e);
        if (lm >= pool || hit[lm]) { std::printf("not a bijection at %llu\n", (unsigned long long)e); return 1; }
        hit[lm] = 1;
        const int block = int(e / (page * layers)), layer = int((e / page) % layers);
        const uint64_t within = e % page;
        const uint64_t slot = within / mpb::kKvWidth, col = within % mpb::kKvWidth;
        // the kernels' layer-major addressing (page_stride 1, layer_offset layer * blocks)
        const uint64_t kernel = (mpb::pool_page(block, 1, int64_t(layer) * blocks) * bt + slot) * mpb::kKvWidth + col;
        if (kernel != lm) { std::printf("kernel address differs at %llu\n", (unsigned long long)e); return 2; }
        // the operator entry points' reference addressing (page_stride layers, layer_offset layer)
        const uint64_t ref = (mpb::pool_page(block, layers, layer) * bt + slot) * mpb::kKvWidth + col;
        if (ref != e) { std::printf("reference address differs at %llu\n", (unsigned long long)e); return 3; }
    }
    // a piece that ends at or before the next reference page boundary is contiguous
    for (uint64_t e = 0; e < pool; e += 4) {
        const uint64_t n = page - e % page, lm = mpb::layer_major_offset(g, e);
        for (uint64_t i = 0; i < n; i += 4)
            if (mpb::layer_major_offset(g, e + i) != lm + i) { std::printf("piece split at %llu\n", (unsigned long long)e); return 4; }
    }
    std::printf("ok\n");
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None or not os.path.isdir(CUDA_INCLUDE),
                    reason="needs g++ and the CUDA headers")
def test_layer_major_translation_matches_kernel_addressing(tmp_path):
    src = tmp_path / "layout_check.cpp"
    src.write_text(CHECKER)
    exe = tmp_path / "layout_check"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{CUDA_INCLUDE}", f"-I{ROOT}/tinyinfer_b200/csrc", str(src), "-o",
                    str(exe)], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
