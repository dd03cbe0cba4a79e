"""KV-state lifetime checking: a ledger of allocations, generations and outstanding asynchronous operations with four
rules (ledger.py), protocol models of prefill/decode and offload serving in buggy and fixed variants (models.py), a
delay-bounded explorer of their event orderings (explore.py), and an adapter that checks a real engine's recorded
events against the same rules (adapter.py).

Reference: src/sdcguard/lifetime/ (ledger.py:1-36, explore.py:1-20, models.py:1-40, adapter.py)."""
