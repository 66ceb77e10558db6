from infera_b200.preflight.cli import main

main()
