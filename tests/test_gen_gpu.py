"""The device generator produces the host generator's bits (GPU)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_matches_host(vc, gpu):
    import torch
    for kind, d in [(vc.GEN_NORMAL, 128), (vc.GEN_NORMAL_UNIT, 128), (vc.GEN_UNIFORM, 96),
                    (vc.GEN_UNIFORM_SUM1, 96), (vc.GEN_NORMAL, 7)]:
        s = vc.config_seed(kind)
        host = vc.gen_rows_host(kind, s, 0, 1000, 4096, d)
        dev = torch.empty((4096, d), dtype=torch.float32, device="cuda")
        vc.gen_rows_device(kind, s, 0, 1000, 4096, d, dev.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(dev.cpu().numpy().view(np.uint32), host.view(np.uint32)), kind
    s = vc.config_seed(2)
    c = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, 64, 32)
    host = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, 2048, 32, c, 64, 0.1)
    dc = torch.from_numpy(c).cuda()
    dev = torch.empty((2048, 32), dtype=torch.float32, device="cuda")
    vc.gen_rows_device(vc.GEN_MIXTURE, s, 0, 0, 2048, 32, dev.data_ptr(), dc.data_ptr(), 64, 0.1)
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy().view(np.uint32), host.view(np.uint32))
