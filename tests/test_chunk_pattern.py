"""Index arithmetic of the 2nd-order code pattern (host-side, no GPU).

The tables kernel writes the 256 codes of each distinct full 2nd-order chunk
(one period of ng / gcd(ng, 256) chunks, at most as many as the matrix has)
in flat order; encode's row writer gives row r < full_rows the codes at
(r mod rp) * ng + g, rp = 256 / gcd(ng, 256).  This checks, for the chunk
layout of core/quantize.cu:245-272 (chunks of 256 over the flattened
[M, ng] scales), that those reads stay inside the pattern and hit the same
chunk position as the row's own flat index r * ng + g."""
import math

import pytest


def layout(M: int, ng: int):
    total = M * ng
    nfull = total // 256
    period = ng // math.gcd(ng, 256)
    ntab_full = min(nfull, period)
    rp = period * 256 // ng
    full_rows = nfull * 256 // ng
    return nfull, period, ntab_full, rp, full_rows


@pytest.mark.parametrize("M,ng", [(4096, 256), (4096, 688), (11008, 256), (28672, 512),
                                  (8192, 1792), (64, 688), (17, 272), (300, 80), (1, 16),
                                  (3, 48), (129, 688), (2, 4096)])
def test_pattern_reads_match_flat_chunks(M, ng):
    nfull, period, ntab_full, rp, full_rows = layout(M, ng)
    assert rp * ng == period * 256
    for r in range(min(full_rows, 3 * rp + 5)):
        for g in range(0, ng, 16):
            e = (r % rp) * ng + g            # the row writer's 16-code read
            assert e + 16 <= ntab_full * 256  # inside what the tables kernel wrote
            si = r * ng + g                  # the flat index of (r, g)
            # both name the same entry of the same distinct chunk
            assert (si % (period * 256)) == e
            assert si + 16 <= nfull * 256    # a full chunk, not the partial one
