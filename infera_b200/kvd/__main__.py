from infera_b200.kvd.server import main

main()
