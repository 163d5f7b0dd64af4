"""CPU oracle of CacheFlow's KV-cache kernel path -- TEST / BENCH INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, always to produce expected results; the cacheflow_b200 package never
imports it.
"""
