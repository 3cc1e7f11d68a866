"""``python -m <package>.server``: the server's command line."""
from .cli import main

main()
