"""``python -m priml_b200 pkg.module.factory [--override ...]``."""

import sys

from priml_b200.launch import main

if __name__ == "__main__":
    sys.exit(main())
