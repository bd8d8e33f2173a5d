from graspo_b200.cli.app import main

main()
