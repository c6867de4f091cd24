"""Host resources of a node: the memory-pressure rule of the reference node (resources.rs:114-129): the
node sheds load when used host memory exceeds its configured fraction plus 10 % of the total."""
from __future__ import annotations


def host_memory_fraction() -> float:
    """Used / total host memory (0.0 when it cannot be read)."""
    try:
        import psutil
        vm = psutil.virtual_memory()
        return float(vm.total - vm.available) / float(vm.total) if vm.total else 0.0
    except Exception:
        pass
    try:
        info = {}
        with open("/proc/meminfo") as f:
            for line in f:
                k, v = line.split(":", 1)
                info[k] = int(v.split()[0])
        return 1.0 - info["MemAvailable"] / info["MemTotal"]
    except Exception:
        return 0.0


def memory_pressure(max_fraction: float = 0.80, used_fraction=None) -> bool:
    used = host_memory_fraction() if used_fraction is None else used_fraction
    return used > min(max_fraction + 0.10, 1.0)
