"""m27b_hbm_read_probe (the benchmark's read ceiling): streams a buffer
through shared memory with bulk copies and returns with every bounded wait
satisfied (status word 0), for sizes that are and are not multiples of the
32 KB chunk and of the SM count; bad arguments are refused."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [16, 4096 + 48, 50135040, 3 * 32768 * 148 + 16 * 7])
def test_probe_streams_and_returns(torch, m27b, nbytes):
    buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    m27b.device_status(clear=True)
    for _ in range(3):
        m27b.hbm_read_probe(buf)
    torch.cuda.synchronize()
    assert m27b.device_status() == 0


def test_probe_rejects_unaligned(torch, m27b):
    buf = torch.empty(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(m27b.M27BError, match="16-byte aligned"):
        m27b.hbm_read_probe(buf[:1000])
