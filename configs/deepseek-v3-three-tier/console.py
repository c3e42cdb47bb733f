"""Console entry: benchmark config 5, the three-tier DeepSeek-V3-shaped decode at 32K context (planner-sized GPU slots,
CPU engine RAM, NVMe cold records, a 4M x 4096 NVMe table in the graph). A run of the measuring tool: it prints one
JSON line with the tiers, tokens per second and the cold-store and table statistics, then exits."""

MODEL = {
    'id': 'deepseek-v3-three-tier', 'order': 30, 'name': 'DeepSeek-V3 shape, three tiers (config 5)', 'port': 18195,
    'ready_timeout': 3600, 'hardware': '1x B200 + host CPU engine + NVMe', 'oneshot': True,
    'options': [
        {'key': 'layers', 'label': 'layers', 'default': '6',
         'choices': [['6', '6 (3 dense + 3 MoE)'], ['12', '12'], ['61', '61 (needs ~260 GB of disk)']]},
        {'key': 'context', 'label': 'context', 'default': '32768', 'choices': [['32768', '32K'], ['8192', '8K']]},
        {'key': 'table', 'label': 'NVMe table', 'default': 'on', 'choices': [['on', '4M x 4096 BF16'], ['off', 'none']]},
    ],
}


def build(options, port):
    """(argv, env) of the tool process for the chosen options."""
    argv = ['python', '-m', 'xtier_b200.tools.three_tier', '--layers', options['layers'], '--context',
            options['context'], '--cold-dir', '/tmp/xtier-cold', '--table-dir', '/tmp/xtier-table']
    if options['table'] == 'off':
        argv.append('--no-table')
    return argv, {}
