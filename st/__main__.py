from exploration_b200.cli import main

main()
