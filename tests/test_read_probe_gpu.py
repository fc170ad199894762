"""m27b_hbm_read_probe / m27b_hbm_read_probe_shape (the benchmark's read
ceiling): streams a buffer through shared memory with bulk copies and
returns with every bounded wait satisfied (status word 0), for sizes that are
and are not multiples of the copy size, of the SM count and of the warps of
the grid, over the shapes the benchmark sweeps; bad arguments and shapes that
do not fit an SM are refused."""
import pytest

pytestmark = pytest.mark.gpu

# (warps, stages, chunk bytes, CTAs per SM); the benchmark's sweep
SHAPES = [None, (8, 2, 4608, 2), (8, 3, 8192, 1), (4, 3, 8192, 2), (16, 2, 4096, 1), (8, 6, 4096, 1)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("nbytes", [16, 4096 + 48, 50135040, 3 * 32768 * 148 + 16 * 7])
def test_probe_streams_and_returns(torch, m27b, nbytes, shape):
    buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    m27b.device_status(clear=True)
    for _ in range(3):
        m27b.hbm_read_probe(buf, shape)
    torch.cuda.synchronize()
    assert m27b.device_status() == 0


def test_probe_rejects_bad_arguments(torch, m27b):
    buf = torch.empty(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(m27b.M27BError, match="16-byte aligned"):
        m27b.hbm_read_probe(buf[:1000])
    for shape in [(0, 2, 4096, 1), (17, 2, 4096, 1), (8, 9, 4096, 1), (8, 2, 4100, 1), (8, 2, 131072, 1),
                  (8, 2, 4096, 0)]:
        with pytest.raises(m27b.M27BError, match="out of range"):
            m27b.hbm_read_probe(buf, shape)
    with pytest.raises(m27b.M27BError, match="do not fit"):
        m27b.hbm_read_probe(buf, (8, 3, 8192, 2))  # 192 KB per CTA: one per SM
    with pytest.raises(m27b.M27BError, match="too many bytes"):
        m27b.hbm_read_probe(buf, (8, 4, 16384, 1))  # 512 KB per CTA
    m27b.hbm_read_probe(buf, (8, 2, 4608, 2))  # a refused shape leaves no error behind
    torch.cuda.synchronize()
    assert m27b.device_status() == 0
