"""Input generators: Philox4x32-10 against the published known-answer vectors."""
import numpy as np

from diskllm_b200.workloads import philox4x32_10, philox_uniforms


def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32-10
    cases = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in cases:
        got = philox4x32_10(np.array([ctr], dtype=np.uint32), key)[0]
        assert tuple(int(x) for x in got) == want


def test_uniforms_on_grid():
    u = philox_uniforms(404, 1000)
    assert u.dtype == np.float32 and np.all((u >= 0) & (u < 1))
    assert np.all((u.astype(np.float64) * 2 ** 24) % 1 == 0)
    assert np.array_equal(u, philox_uniforms(404, 1000))
