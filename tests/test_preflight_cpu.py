"""Pre-flight probe pieces that need no GPU: NVLink link counting against a
fake NVML, and the no-CUDA report."""
import importlib

pf = importlib.import_module("3080_mod_p2p_sglang_patch_b200.utils.preflight")


class FakeNVML:
    NVML_NVLINK_MAX_LINKS = 18
    NVML_FEATURE_ENABLED = 1

    class NVMLError(Exception):
        pass

    def __init__(self, links):
        self.links = links  # per device: list of link states; past the end -> NVMLError
        self.inited = 0

    def nvmlInit(self):
        self.inited += 1

    def nvmlShutdown(self):
        self.inited -= 1

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= len(self.links[h]):
            raise self.NVMLError("no such link")
        return self.links[h][link]


def test_nvlink_links_counted_and_nvml_shut_down():
    fake = FakeNVML([[1] * 18, [1] * 16 + [0, 0], [0] * 4])
    assert pf.nvlink_links_up(3, nvml=fake) == [18, 16, 0]
    assert fake.inited == 0


def test_nvml_failure_is_reported_not_raised():
    class Broken(FakeNVML):
        def nvmlInit(self):
            raise RuntimeError("driver not loaded")

    assert pf.nvlink_links_up(2, nvml=Broken([])).startswith("unknown")


def test_preflight_without_cuda(monkeypatch):
    monkeypatch.setattr(pf.torch.cuda, "is_available", lambda: False)
    assert pf.preflight() == {"cuda": False, "devices": 0}
