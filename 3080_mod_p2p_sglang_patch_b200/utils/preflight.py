"""Pre-flight probe of a node: device count, P2P access matrix, multicast
(NVLS) support. Replaces the reference's bring-up script
(scripts/sglang-p2p.sh: driver swap, FLR, readiness probe, watchdog), none of
which applies to shared B200 nodes: nothing here changes driver or GPU state."""
import json

import torch


def preflight() -> dict:
    info = {"cuda": torch.cuda.is_available(), "devices": 0}
    if not info["cuda"]:
        return info
    n = torch.cuda.device_count()
    info["devices"] = n
    info["names"] = [torch.cuda.get_device_name(i) for i in range(n)]
    info["capability"] = [list(torch.cuda.get_device_capability(i)) for i in range(n)]
    info["p2p"] = [[(i == j) or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)] for i in range(n)]
    try:
        from .._ext import cuda_ext

        C = cuda_ext()
        info["multicast"] = [bool(C.mc_supported(i)) for i in range(n)]
    except Exception as e:  # noqa: BLE001
        info["multicast"] = f"unknown ({e})"
    return info


if __name__ == "__main__":
    print(json.dumps(preflight(), indent=1))
