"""CPU oracle for the KML operator set -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline
legs as the checker of the CUDA path; the product library never imports it.
"""
from .oracle import *  # noqa: F401,F403
