import sys

from difflet_b200.cli.main import main

sys.exit(main())
