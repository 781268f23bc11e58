import sys

from meshtrain_b200.cli import main

sys.exit(main())
