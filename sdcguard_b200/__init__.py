"""sdcguard_b200: a Blackwell-native (sm_100a) guard against silent data corruption in LLM serving and training.

Every checked hot path is a hand-written sm_100a CUDA kernel that fuses its check into the work it guards
(checked GEMMs with ABFT epilogues, checksummed KV-block transfer, checksummed all-to-all, sampled attention
recompute). The Python layer keeps the `sdcguard` CLI, the checksum-record schema and the offline coverage gate.
"""
__version__ = "0.1.0"
