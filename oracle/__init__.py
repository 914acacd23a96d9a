"""CPU oracle and reference checker of the r2splat hot path (test infrastructure only)."""
import os

# Where a BT-3DGS checkout is looked for when the checker is built or the
# golden fixtures are regenerated; absent on machines that only run tests.
REFERENCE_ROOT = os.environ.get("BT3DGS_REFERENCE_ROOT", "/root/reference")
