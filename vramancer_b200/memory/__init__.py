"""Memory tiers beyond the KV pool: hierarchical block store (VRAM -> peer VRAM ->
pinned DRAM -> NVMe -> archive / remote), XOR parity groups, byte / tensor
compression."""
from .compressor import Compressor
from .hierarchy import HierarchicalMemoryManager, MemoryBlock, Tier
from .parity import ParityKVManager

__all__ = ["Compressor", "HierarchicalMemoryManager", "MemoryBlock", "ParityKVManager", "Tier"]
