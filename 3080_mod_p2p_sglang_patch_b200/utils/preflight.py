"""Pre-flight probe of a node: device count, P2P access matrix, multicast
(NVLS) support. Replaces the reference's bring-up script
(scripts/sglang-p2p.sh: driver swap, FLR, readiness probe, watchdog), none of
which applies to shared B200 nodes: nothing here changes driver or GPU state."""
import json

import torch


def nvlink_links_up(n: int, nvml=None):
    """Active NVLink links per device through NVML (read-only), or a string
    saying why they could not be read. ``nvml`` defaults to pynvml."""
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        try:
            out = []
            for i in range(n):
                h = nvml.nvmlDeviceGetHandleByIndex(i)
                up = 0
                for link in range(nvml.NVML_NVLINK_MAX_LINKS):
                    try:
                        if nvml.nvmlDeviceGetNvLinkState(h, link) == nvml.NVML_FEATURE_ENABLED:
                            up += 1
                    except nvml.NVMLError:
                        break  # no more links on this device
                out.append(up)
            return out
        finally:
            nvml.nvmlShutdown()
    except Exception as e:  # noqa: BLE001
        return f"unknown ({e})"


def cuda_ready(n: int):
    """Per device: a tiny allocation and a synchronize succeed (the
    reference's readiness probe, scripts/sglang-p2p.sh:34-54)."""
    out = []
    for i in range(n):
        try:
            torch.zeros(1, device=f"cuda:{i}")
            torch.cuda.synchronize(i)
            out.append(True)
        except Exception:  # noqa: BLE001
            out.append(False)
    return out


def preflight() -> dict:
    info = {"cuda": torch.cuda.is_available(), "devices": 0}
    if not info["cuda"]:
        return info
    n = torch.cuda.device_count()
    info["devices"] = n
    info["names"] = [torch.cuda.get_device_name(i) for i in range(n)]
    info["capability"] = [list(torch.cuda.get_device_capability(i)) for i in range(n)]
    info["ready"] = cuda_ready(n)
    info["p2p"] = [[(i == j) or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)] for i in range(n)]
    info["nvlink_links_up"] = nvlink_links_up(n)
    try:
        from .._ext import cuda_ext

        C = cuda_ext()
        info["multicast"] = [bool(C.mc_supported(i)) for i in range(n)]
    except Exception as e:  # noqa: BLE001
        info["multicast"] = f"unknown ({e})"
    return info


if __name__ == "__main__":
    print(json.dumps(preflight(), indent=1))
