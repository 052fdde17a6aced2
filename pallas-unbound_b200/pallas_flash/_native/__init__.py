"""Directory of the built sm_100a library (libpu_attn.so), produced by
pallas-unbound_b200/build.py."""
