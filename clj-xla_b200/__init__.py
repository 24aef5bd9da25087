"""clj-xla B200 executor: the PJRT plugin library ``libcljxla_b200.so`` and a
host-side mirror of the clj-xla API that drives it."""
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libcljxla_b200.so")
