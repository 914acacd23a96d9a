"""CPU oracle and reference checker of the r2splat hot path (test infrastructure only)."""
import os

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Where a BT-3DGS checkout is looked for when the checker is built or the
# golden fixtures are regenerated: the BT3DGS_REFERENCE_ROOT environment
# variable, else a checkout named "reference" beside this repository.  Absent
# on machines that only run tests (they use the prebuilt checker and the
# committed fixtures).
REFERENCE_ROOT = (os.environ.get("BT3DGS_REFERENCE_ROOT")
                  or os.path.normpath(os.path.join(_REPO, os.pardir, "reference")))
