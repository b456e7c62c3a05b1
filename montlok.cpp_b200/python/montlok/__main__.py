"""`python -m montlok` runs the `montlok` command."""

import sys

from .cli import main

sys.exit(main())
