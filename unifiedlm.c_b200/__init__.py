"""B200-native (sm_100a) fast-memory path of UnifiedLM.

Modules mirror the reference's layout (ruhai-lin/unifiedlm.c):
  kernel  - unified_memory / UnifiedMemory, the fast-memory operator (kernel.py)
  export  - model.bin v1 reader/writer (export.py, run.c's checkpoint format)
The compute runs in libulm_b200.so, whose C ABI is include/ulm_b200.h.
"""
import os

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
